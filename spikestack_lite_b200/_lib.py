"""ctypes binding of libspk_b200.so (declared in include/spikestack_b200.h).

This is the FFI a Python host uses for the engine: every call passes raw
device pointers, sizes and the current CUDA stream of the tensors' device.
A missing library or a non-CUDA tensor is an error -- there is no CPU path.
"""
import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libspk_b200.so")

SPK_OK, SPK_EINVAL, SPK_EUNSUPPORTED, SPK_ECUDA, SPK_EWORKSPACE, SPK_EDEVICE = range(6)
SPK_F32, SPK_BF16 = 0, 1
# device error bits (spk_device_error)
SPK_DEV_PIPE_TIMEOUT, SPK_DEV_SCAN_TIMEOUT, SPK_DEV_CSR_OVERFLOW, SPK_DEV_TMEM = 1, 2, 4, 8
BRANCH_AUTO, BRANCH_DENSE, BRANCH_CSR = 0, 1, 2
BRANCHES = {"auto": BRANCH_AUTO, "dense": BRANCH_DENSE, "csr": BRANCH_CSR}

_c = ctypes
_P, _I, _L, _F, _Z = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_float, _c.c_size_t

# name -> (restype, argtypes); the order follows include/spikestack_b200.h
SIGNATURES = {
    "spk_last_error": (_c.c_char_p, []),
    "spk_version": (_I, []),
    "spk_device_error": (_I, [_I, _c.POINTER(_I)]),
    "spk_timeout_site": (_I, [_c.POINTER(_c.c_uint64)]),
    "spk_launch_count": (_L, []),
    "spk_profile_begin": (_I, [_I]),
    "spk_profile_end": (_I, [_c.POINTER(_c.c_double), _c.POINTER(_L)]),
    "spk_csr_workspace_bytes": (_Z, [_I, _L, _I]),
    "spk_csr_compact": (_I, [_P, _I, _L, _I, _P, _P, _P, _P, _P, _L, _P, _Z, _P]),
    "spk_csr_compact_noalloc": (_I, [_P, _I, _L, _I, _P, _P, _P, _P, _P, _L, _P]),
    "spk_spike_linear_workspace_bytes": (_Z, [_I, _L, _I, _I, _I]),
    "spk_linear_act_workspace_bytes": (_Z, [_I, _I]),
    "spk_linear_act": (_I, [_P, _L, _I, _P, _L, _L, _I, _P, _I, _F, _P, _P, _Z, _P]),
    "spk_spike_linear": (_I, [_P, _I, _L, _I, _P, _I, _L, _L, _I, _P, _P, _P, _P, _P, _P, _P, _L, _I, _P, _Z, _P]),
    "spk_weight_image_bytes": (_Z, [_I, _I, _I]),
    "spk_weight_image": (_I, [_P, _I, _L, _L, _I, _I, _P, _Z, _P]),
    "spk_spike_linear_img": (_I, [_P, _I, _L, _I, _P, _I, _L, _L, _I, _P, _P, _P, _P, _P, _P, _P, _P, _L, _I, _P, _Z,
                                  _P]),
    "spk_linear_act_img": (_I, [_P, _L, _I, _P, _L, _L, _I, _P, _P, _I, _F, _P, _P, _Z, _P]),
    "spk_spike_linear_bits": (_I, [_P, _I, _L, _I, _P, _L, _L, _I, _P, _P, _P, _P, _Z, _P]),
    "spk_sparse_forward_workspace_bytes": (_Z, [_I, _L, _I, _I]),
    "spk_sparse_forward": (_I, [_P, _L, _I, _P, _I, _P, _P, _P, _P, _L, _P, _I, _P, _Z, _P]),
    "spk_sparse_multistep_forward": (_I, [_P, _I, _L, _I, _P, _I, _P, _P, _P, _P, _L, _P, _I, _P, _Z, _P]),
    "spk_apply_channel_decay": (_I, [_P, _P, _L, _I, _I, _P, _P]),
    "spk_normalize_attention": (_I, [_P, _P, _L, _F, _P, _P]),
    "spk_attention_workspace_bytes": (_Z, [_L, _I, _I, _I]),
    "spk_spiking_attention": (_I, [_P, _P, _P, _P, _L, _I, _I, _I, _F, _P, _P, _Z, _P]),
    "spk_spiking_attention_bits": (_I, [_P, _P, _P, _P, _L, _I, _I, _I, _F, _P, _P, _Z, _P]),
    "spk_gsmc_step": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _L, _I, _F, _F, _I, _F, _P]),
    "spk_gsmc_workspace_bytes": (_Z, [_L, _I]),
    "spk_gsmc_forward": (_I, [_P, _P, _P, _P, _I, _L, _I, _F, _F, _I, _F, _I, _P, _P, _P, _Z, _P]),
    "spk_gsmc_forward_ex": (_I, [_P, _P, _P, _P, _I, _L, _I, _F, _F, _I, _F, _I, _P, _P, _P, _Z, _I, _P]),
    "spk_add_layernorm": (_I, [_P, _P, _P, _P, _L, _I, _F, _P, _P, _P]),
    "spk_selftest_wait_timeout": (_I, [_P]),
    "spk_spire_planes": (_I, [_P, _P, _P, _P, _I, _L, _I, _I, _P, _P]),
    "spk_temporal_mean": (_I, [_P, _I, _L, _I, _I, _P, _P, _P]),
}

_lib = None
_lock = threading.Lock()


class EngineError(RuntimeError):
    """An engine entry point returned an error status."""


def load():
    """Load libspk_b200.so and declare every entry point; raises when absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise EngineError(
                    f"spikestack_lite_b200: {LIB_PATH} is not built "
                    "(run `python -m spikestack_lite_b200.build`)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc, what):
    if rc != SPK_OK:
        msg = load().spk_last_error().decode(errors="replace")
        raise EngineError(f"{what}: {msg} (status {rc})")


def ptr(t):
    return None if t is None else t.data_ptr()


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors, what="spikestack_lite_b200"):
    for t in tensors:
        if t is not None and (not isinstance(t, torch.Tensor) or t.device.type != "cuda"):
            raise EngineError(f"{what}: CUDA tensors required (this engine has no CPU path)")


def require_f32(*tensors, what="spikestack_lite_b200"):
    for t in tensors:
        if t is not None and t.dtype != torch.float32:
            raise EngineError(f"{what}: float32 tensors required, got {t.dtype}")


class _Workspaces:
    """One grow-only scratch buffer per device (the engine keeps no state in it)."""

    def __init__(self):
        self._bufs = {}
        self._lock = threading.Lock()

    def get(self, device, nbytes):
        idx = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            buf = self._bufs.get(idx)
            if buf is None or buf.numel() < nbytes:
                size = max(int(nbytes), 1 << 20)
                if buf is not None:
                    size = max(size, int(buf.numel() * 1.25))
                buf = torch.empty(size, dtype=torch.uint8, device=torch.device("cuda", idx))
                self._bufs[idx] = buf
            return buf

    def clear(self):
        with self._lock:
            self._bufs.clear()


workspaces = _Workspaces()


def workspace(device, nbytes):
    buf = workspaces.get(device, nbytes)
    return ctypes.c_void_p(buf.data_ptr()), buf.numel()


def launch_count():
    return int(load().spk_launch_count())


KERNELS = {"dense": 1, "csr_scan": 2, "spmm_csr": 3, "attn_kv": 4, "attn_out": 5, "gsmc_step": 6, "w_image": 7}


def profile_begin(kernel):
    check(load().spk_profile_begin(KERNELS[kernel]), "spk_profile_begin")


def profile_end():
    """(summed device milliseconds, launches) of the profiled kernel."""
    ms = ctypes.c_double(0.0)
    n = ctypes.c_int64(0)
    check(load().spk_profile_end(ctypes.byref(ms), ctypes.byref(n)), "spk_profile_end")
    return ms.value, n.value


def device_error(clear=True):
    bits = ctypes.c_int(0)
    check(load().spk_device_error(1 if clear else 0, ctypes.byref(bits)), "spk_device_error")
    return bits.value


def timeout_site():
    """(block, warp, mbarrier shared address) of the first timed-out pipeline wait, or None."""
    site = ctypes.c_uint64(0)
    check(load().spk_timeout_site(ctypes.byref(site)), "spk_timeout_site")
    v = site.value
    return None if v == 0 else (v >> 40, (v >> 32) & 0xff, v & 0xffffffff)
