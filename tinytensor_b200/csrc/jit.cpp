// Kernel compilation for generated regions: NVRTC straight to an sm_100a CUBIN,
// a disk cache keyed by SHA-256, and module loading through driver entry points
// obtained from the runtime (so the library itself does not link libcuda).
//
// The cache keeps the reference KernelCache protocol (src/codegen/kernel_cache.cpp):
//   key   = SHA-256(version, ABI/flags line, compiler info, IR, metadata)  (:190-202)
//   get   = exists, size >= 64, ELF magic, else evict                     (:204-242)
//   put   = write a temp file, then rename under a per-key flock          (:260-313)
//   compile under a per-key compile lock, re-checking the cache after it  (cpp_backend.cpp:596-628)
// A cubin is an ELF image, so the same integrity checks apply.
#include <cuda.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <nvrtc.h>
#include <sys/file.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <mutex>
#include <sstream>

#include "jit.hpp"

namespace ttb {

namespace {

std::atomic<uint64_t> g_hits{0}, g_misses{0};
std::mutex g_cache_mutex;

template <typename F>
F entry(const char* name) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        fail(TT_ERR_NO_DEVICE, std::string("CUDA driver entry point unavailable: ") + name);
    return reinterpret_cast<F>(fn);
}

struct FileLock {
    int fd = -1;
    explicit FileLock(const std::string& path) {
        fd = ::open(path.c_str(), O_CREAT | O_RDWR, 0666);
        if (fd >= 0 && ::flock(fd, LOCK_EX) != 0) {
            ::close(fd);
            fd = -1;
        }
    }
    ~FileLock() {
        if (fd >= 0) {
            ::flock(fd, LOCK_UN);
            ::close(fd);
        }
    }
};

bool read_valid_cubin(const std::string& path, std::string& out) {
    namespace fs = std::filesystem;
    std::error_code ec;
    if (!fs::exists(path, ec)) return false;
    auto sz = fs::file_size(path, ec);
    if (ec || sz < 64) {
        fs::remove(path, ec);
        return false;
    }
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::string data((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (data.size() < 64 || static_cast<unsigned char>(data[0]) != 0x7f || data[1] != 'E' || data[2] != 'L' ||
        data[3] != 'F') {
        fs::remove(path, ec);
        return false;
    }
    out = std::move(data);
    return true;
}

void publish(const std::string& dir, const std::string& key, const std::string& ext, const std::string& data) {
    namespace fs = std::filesystem;
    std::error_code ec;
    FileLock lock(dir + "/" + key + ".publish.lock");
    std::string final_path = dir + "/" + key + ext;
    if (ext == ".cubin" && fs::exists(final_path, ec) && fs::file_size(final_path, ec) >= 64) return;
    std::ostringstream tmp;
    tmp << dir << "/" << key << ".tmp." << ::getpid() << "."
        << std::chrono::steady_clock::now().time_since_epoch().count() << ext;
    {
        std::ofstream f(tmp.str(), std::ios::binary);
        if (!f) return;
        f.write(data.data(), static_cast<std::streamsize>(data.size()));
        if (!f) {
            f.close();
            fs::remove(tmp.str(), ec);
            return;
        }
    }
    fs::rename(tmp.str(), final_path, ec);
    if (ec) fs::remove(tmp.str(), ec);
}

}  // namespace

const Driver& driver() {
    static Driver d = [] {
        Driver x;
        x.moduleLoadData = entry<PFN_cuModuleLoadData_v2000>("cuModuleLoadData");
        x.moduleGetFunction = entry<PFN_cuModuleGetFunction_v2000>("cuModuleGetFunction");
        x.moduleUnload = entry<PFN_cuModuleUnload_v2000>("cuModuleUnload");
        x.launchKernel = entry<PFN_cuLaunchKernel_v4000>("cuLaunchKernel");
        x.tensorMapEncodeTiled = entry<PFN_cuTensorMapEncodeTiled_v12000>("cuTensorMapEncodeTiled");
        x.getErrorString = entry<PFN_cuGetErrorString_v6000>("cuGetErrorString");
        return x;
    }();
    return d;
}

std::string cu_error(CUresult r) {
    const char* s = nullptr;
    if (driver().getErrorString(r, &s) != CUDA_SUCCESS || !s) return "CUresult " + std::to_string(static_cast<int>(r));
    return s;
}

std::string nvrtc_info() {
    int major = 0, minor = 0;
    nvrtcVersion(&major, &minor);
    return "nvrtc-" + std::to_string(major) + "." + std::to_string(minor) + " sm_100a --fmad=false";
}

static const char* kNvrtcOptions[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--std=c++17",
                                      "-default-device", "--device-as-default-execution-space"};

std::string nvrtc_compile(const std::string& source) {
    nvrtcProgram prog;
    if (nvrtcCreateProgram(&prog, source.c_str(), "tt_program.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
        fail(TT_ERR_COMPILE, "nvrtcCreateProgram failed");
    nvrtcResult r = nvrtcCompileProgram(prog, 4, kNvrtcOptions);
    if (r != NVRTC_SUCCESS) {
        size_t n = 0;
        nvrtcGetProgramLogSize(prog, &n);
        std::string log(n, '\0');
        if (n) nvrtcGetProgramLog(prog, &log[0]);
        nvrtcDestroyProgram(&prog);
        fail(TT_ERR_COMPILE, std::string("Kernel compilation failed (") + nvrtcGetErrorString(r) + "):\n" + log);
    }
    size_t n = 0;
    nvrtcGetCUBINSize(prog, &n);
    std::string cubin(n, '\0');
    if (n == 0 || nvrtcGetCUBIN(prog, &cubin[0]) != NVRTC_SUCCESS) {
        nvrtcDestroyProgram(&prog);
        fail(TT_ERR_COMPILE, "NVRTC produced no CUBIN");
    }
    nvrtcDestroyProgram(&prog);
    return cubin;
}

std::string cache_key(const std::string& canonical_ir, const std::string& metadata) {
    std::string s;
    s += "tinytensor_b200_v0.1.0\n";
    s += "abi=tt_program_run_v1;arch=sm_100a;flags=--fmad=false,-default-device\n";
    s += nvrtc_info();
    s += "\n---IR---\n";
    s += canonical_ir;
    s += "\n---META---\n";
    s += metadata;
    return sha256_hex(s);
}

uint64_t cache_hits() { return g_hits.load(); }

std::string compile_to_cache(const std::string& key, const std::string& source, const std::string& cache_dir) {
    namespace fs = std::filesystem;
    std::string cubin;
    if (cache_dir.empty()) {
        g_misses++;
        nvrtc_compile(source);
        return "";
    }
    std::error_code ec;
    fs::create_directories(cache_dir, ec);
    std::string path = cache_dir + "/" + key + ".cubin";
    if (read_valid_cubin(path, cubin)) {
        g_hits++;
        return path;
    }
    FileLock compile_lock(cache_dir + "/" + key + ".compile.lock");
    if (read_valid_cubin(path, cubin)) {
        g_hits++;
        return path;
    }
    g_misses++;
    cubin = nvrtc_compile(source);
    publish(cache_dir, key, ".cubin", cubin);
    publish(cache_dir, key, ".cu", source);
    return path;
}
uint64_t cache_misses() { return g_misses.load(); }

LoadedModule load_program_module(const std::string& key, const std::string& source, const std::string& cache_dir,
                                 const std::vector<std::string>& kernels) {
    namespace fs = std::filesystem;
    LoadedModule m;
    std::string cubin;
    bool from_cache = false;
    auto try_load = [&](const std::string& image) -> bool {
        CUmodule mod = nullptr;
        CUresult r = driver().moduleLoadData(&mod, image.data());
        if (r != CUDA_SUCCESS) return false;
        std::vector<CUfunction> fns;
        for (const std::string& k : kernels) {
            CUfunction f = nullptr;
            if (driver().moduleGetFunction(&f, mod, k.c_str()) != CUDA_SUCCESS) {
                driver().moduleUnload(mod);
                return false;
            }
            fns.push_back(f);
        }
        m.module = mod;
        m.functions = std::move(fns);
        return true;
    };
    if (!cache_dir.empty()) {
        std::error_code ec;
        fs::create_directories(cache_dir, ec);
        std::string path = cache_dir + "/" + key + ".cubin";
        {
            std::lock_guard<std::mutex> lk(g_cache_mutex);
            from_cache = read_valid_cubin(path, cubin);
        }
        if (from_cache && try_load(cubin)) {
            g_hits++;
            m.cubin_path = path;
            m.from_cache = true;
            return m;
        }
        if (from_cache) fs::remove(path, ec);  // valid ELF header but unusable: heal
        FileLock compile_lock(cache_dir + "/" + key + ".compile.lock");
        if (read_valid_cubin(path, cubin) && try_load(cubin)) {  // another process finished it
            g_hits++;
            m.cubin_path = path;
            m.from_cache = true;
            return m;
        }
        g_misses++;
        cubin = nvrtc_compile(source);
        publish(cache_dir, key, ".cubin", cubin);
        publish(cache_dir, key, ".cu", source);
        m.cubin_path = path;
    } else {
        g_misses++;
        cubin = nvrtc_compile(source);
    }
    if (!try_load(cubin)) fail(TT_ERR_COMPILE, "cuModuleLoadData rejected the compiled CUBIN");
    return m;
}

}  // namespace ttb
