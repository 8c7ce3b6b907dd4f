"""SGD with the reference API (python/tinytensor/optim.py:6-35), on device.

The reference updates host tensors through numpy; here parameters, gradients and
velocities are device buffers and one fused kernel (tt_sgd_step) updates them all:
    v = momentum*v + g   (momentum > 0)
    p = p - lr * (v or g)
in float32, the same arithmetic numpy performs for the reference.
"""

import ctypes

from . import _lib
from ._lib import TypeError
from .compiler import DeviceBuffer, Stream

__all__ = ["SGD"]


class SGD:
    def __init__(self, params, lr: float = 0.01, momentum: float = 0.0):
        for p in params:
            if not isinstance(p, DeviceBuffer):
                raise TypeError("SGD on the CUDA backend updates DeviceBuffer parameters")
        self.params = list(params)
        self.lr = float(lr)
        self.momentum = float(momentum)
        self.velocities = []
        if self.momentum > 0.0:
            for p in self.params:
                v = DeviceBuffer(p.shape)
                _zero = bytes(v.nbytes)
                _lib.check(_lib.lib.tt_memcpy(v.ptr, _zero, v.nbytes, _lib.H2D, None))
                self.velocities.append(v)
        n = len(self.params)
        self._p = (ctypes.c_void_p * max(1, n))(*[p.ptr for p in self.params])
        self._v = (ctypes.c_void_p * max(1, n))(*[v.ptr for v in self.velocities]) if self.velocities else None
        self._n = (ctypes.c_int64 * max(1, n))(*[p.nbytes // 4 for p in self.params])

    def step_one(self, i: int, grad, stream=None, lr_scale: float = 1.0) -> None:
        """Queues the update of parameter i alone (same arithmetic as step)."""
        gp = (ctypes.c_void_p * 1)(getattr(grad, "ptr", grad))
        pp = (ctypes.c_void_p * 1)(self.params[i].ptr)
        vp = (ctypes.c_void_p * 1)(self.velocities[i].ptr) if self.velocities else None
        nn = (ctypes.c_int64 * 1)(self.params[i].nbytes // 4)
        h = stream.handle if isinstance(stream, Stream) else stream
        _lib.check(_lib.lib.tt_sgd_step(1, pp, gp, vp, nn, ctypes.c_float(self.lr * lr_scale),
                                        ctypes.c_float(self.momentum), h))

    def step(self, grads, stream=None, lr_scale: float = 1.0) -> None:
        """Queues the update on `stream`; lr_scale folds e.g. 1/world for data parallel."""
        if len(grads) != len(self.params):
            raise ValueError("one gradient per parameter is required")
        gp = (ctypes.c_void_p * max(1, len(grads)))(*[getattr(g, "ptr", g) for g in grads])
        h = stream.handle if isinstance(stream, Stream) else stream
        _lib.check(_lib.lib.tt_sgd_step(len(self.params), self._p, gp, self._v, self._n,
                                        ctypes.c_float(self.lr * lr_scale), ctypes.c_float(self.momentum), h))
