"""Helpers for the GPU tests: device buffers through the C ABI, and the oracle
comparison used by every parity test."""
import ctypes as C

import numpy as np

import ti_b200 as ti
from oracle import bf16_to_f32

# the benchmark tolerance for bf16 logits: max|y - y_ref| / max|y_ref| <= 2e-2
LOGIT_TOL = 2e-2


class DevBuf:
    def __init__(self, nbytes, device=0):
        p = C.c_void_p()
        ti.check(ti.lib().ti_malloc(device, max(16, nbytes), C.byref(p)))
        self.ptr = p.value
        self.nbytes = nbytes
        self.device = device

    @classmethod
    def from_array(cls, a, device=0):
        a = np.ascontiguousarray(a)
        b = cls(a.nbytes, device)
        ti.check(ti.lib().ti_memcpy_h2d(b.ptr, a.ctypes.data_as(C.c_void_p), a.nbytes, None))
        return b

    def to_array(self, shape, dtype):
        out = np.empty(shape, dtype)
        ti.check(ti.lib().ti_memcpy_d2h(out.ctypes.data_as(C.c_void_p), self.ptr, out.nbytes, None))
        return out

    def free(self):
        if self.ptr:
            ti.lib().ti_free(self.device, self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def top2_margin(lf):
    s = np.sort(lf)
    return float(s[-1] - s[-2])


def check_step(ids_gpu, lb_gpu, lf_ref, what=""):
    """one sequence, one step: bf16 logits within LOGIT_TOL; greedy id equal unless
    the oracle's top-2 margin is below the logits' own error (a recorded near-tie)"""
    g = bf16_to_f32(lb_gpu)
    err = rel_err(g, lf_ref)
    assert err <= LOGIT_TOL, f"{what}: logits rel err {err:.3e}"
    ref_id = int(np.argmax(lf_ref))
    if ids_gpu != ref_id:
        margin = top2_margin(lf_ref)
        noise = float(np.abs(g - lf_ref).max())
        assert margin <= 2 * noise, f"{what}: greedy id {ids_gpu} != {ref_id} with margin {margin:.3e} > noise {noise:.3e}"
        return False
    return True
