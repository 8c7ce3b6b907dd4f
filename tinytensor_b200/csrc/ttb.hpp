// Internal declarations of libtt_cuda.so (the B200 backend behind include/tt_cuda.h).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "tt_cuda.h"

namespace ttb {

using Shape = std::vector<int64_t>;

// ---- errors: one class carrying a tt_status, mapped to the reference exception names ----
struct Error : std::runtime_error {
    int status;
    Error(int st, const std::string& msg) : std::runtime_error(msg), status(st) {}
};
[[noreturn]] void fail(int status, const std::string& msg);
// Sets the thread's tt_last_error() message for a status returned without throwing.
int record_error(int status, const std::string& msg);

// ---- graph (C++ image of tinytensor::Graph, include/tinytensor/graph/graph.hpp) ----
struct Node {
    int op = TT_OP_INPUT;
    int dtype = TT_FLOAT32;
    std::vector<int> in;
    Shape shape;
    int64_t id = 0;
    int64_t dim0 = 0, dim1 = 0;
    std::vector<int64_t> axes;
    bool keepdims = false;
    std::vector<float> cdata;  // Constant payload (float32)
    std::string name, expr;
    // Set by the scheduler only: a matmul's epilogue activation (program.hpp Epilogue),
    // and on that activation node the index of the matmul that computes it.
    int epilogue = 0;
    int fused_into = -1;
    // Set by the scheduler only: a matmul with K <= 16 evaluated inside the fused region
    // of its elementwise readers (no GEMM launch, no stored product).
    bool inline_mm = false;
};

struct Graph {
    std::vector<Node> nodes;
    std::vector<int> inputs;   // graph-input order
    std::vector<int> outputs;  // graph-output order
    int64_t next_id = 0;

    int add(Node n);  // appends, assigns id = next_id++ unless n.id >= next_id
};

int64_t numel(const Shape& s);
std::string shape_str(const Shape& s);  // "[4, 4]"
Shape broadcast_shapes(const Shape& a, const Shape& b);  // throws TT_ERR_BROADCAST
std::vector<int64_t> normalized_axes(const Node& n, int64_t in_rank);  // sorted, unique
const char* op_name(int op);
bool is_elementwise(int op);
bool is_view(int op);
bool is_reduce(int op);

// graph.cpp
Graph import_graph(const tt_graph* g);
void infer_shape(Graph& g, Node& n);  // sets n.shape from inputs/attrs, throws on bad shapes
void verify(const Graph& g);          // src/ir/verifier.cpp rules
std::string ir_text(const Graph& g);  // src/ir/printer.cpp format
Graph expand_fused(const Graph& g);   // FusedElementwise -> primitive nodes
Graph dce(const Graph& g, size_t* removed);
Graph cse(const Graph& g, size_t* removed);

// autodiff.cpp: appends the backward graph and the gradient outputs
void append_gradients(Graph& g, int loss, const std::vector<int>& wrt);

// sha256.cpp
std::string sha256_hex(const std::string& data);

}  // namespace ttb
