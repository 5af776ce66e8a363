"""ctypes binding of ``libdan_b200.so`` (the C ABI declared in include/dan_b200.h).

Arguments are raw device pointers, strides in elements and plain integers; the
stream is the current torch CUDA stream. A non-zero return code raises
``RuntimeError`` with the library's error text. There is no fallback: when the
library is missing or no GPU is present, the first call fails loudly.
"""
import ctypes
import os

import torch

from . import profiling

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdan_b200.so")

P, I64, I32, F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

SIGNATURES = {
    "dan_version": ([], ctypes.c_char_p),
    "dan_last_error": ([], ctypes.c_char_p),
    "dan_read_status": ([P, P, P], I32),
    "dan_selftest_wait": ([I32, P, P, P], I32),
    "dan_gemm_bf16": ([P, I64, P, I64, P, I64, P, I64, P, I32, I32, I32, I32, P, P], I32),
    "dan_gemm_bf16_noalloc": ([P, I64, P, I64, P, I64, P, I64, P, I32, I32, I32, I32, P, P], I32),
    "dan_gemm_e4m3": ([P, I64, P, P, I64, P, P, I64, P, I64, P, I32, I32, I32, I32, P, P], I32),
    "dan_gemm_bf16_rope": ([P, I64, P, I64, P, I64, P, I64, P, I32, I32, I32, I32, I32, I32, P, P, P, P], I32),
    "dan_gemm_e4m3_rope": ([P, I64, P, P, I64, P, P, I64, P, I64, P, I32, I32, I32, I32, I32, I32, P, P, P, P],
                           I32),
    "dan_rope_table": ([P, P, I32, I32, P, P, P], I32),
    "dan_tree_attention": ([P, I64, I64, P, I64, I64, P, I64, I64, P, P, I64, I64, I32, P, I64, I64, I32, I32, I32,
                            I32, P, I32, P, P, P, I32, F32, P, P], I32),
    "dan_embed": ([P, P, I64, I64, P, I64, I32, I32, P, P], I32),
    "dan_rms_norm": ([P, I64, I64, I32, P, F32, I32, P, I64, I64, P, I64, P, I32, I32, P], I32),
    "dan_quantize_e4m3": ([P, I64, P, I64, P, I32, I32, P], I32),
    "dan_rope": ([P, I64, I64, I32, I32, I32, P, P, I32, P], I32),  # x, ld_row, ld_head, heads, d, rot, cos, sin
    "dan_sigmoid_gate": ([P, I64, P, I64, I64, I32, I32, I32, P], I32),
    "dan_kv_store": ([P, P, I64, I64, P, P, I64, I64, P, P, I32, I32, I32, P], I32),
    "dan_label_readout": ([P, I64, P, P, F32, I32, P, I64, I64, P, P, I32, I32, I32, P, P, P, P], I32),
    "dan_causal_conv": ([P, I64, P, I64, P, P, P, I64, I32, I32, P], I32),
    "dan_gather_rows": ([P, I64, P, I64, P, I32, P, I64, I32, P], I32),
    "dan_gated_delta_scan": ([P, P, P, I64, P, P, I64, P, P, P, I32, P, P, I32, P, I64, P, I64, I32, I32, I32, I32,
                              F32, P, I64, I32, I32, P, P], I32),
    "dan_gated_delta_scratch_bytes": ([I32, I32, I32], I64),
    "dan_gated_rms_norm": ([P, I64, P, I64, P, F32, P, I64, I32, I32, I32, P], I32),
    "dan_delta_rule_scan": ([P, P, P, I64, P, I64, P, I64, P, I32, P, P, I32, P, I64, P, I64, I32, I32, I32, I32, F32,
                             P, I64, P, P], I32),
    "dan_swiglu": ([P, I64, P, I64, P, I64, I32, I32, P], I32),
    "dan_delta_gates": ([P, I64, P, I64, P, P, P, I64, P, I64, I32, I32, P], I32),
    "dan_lse_merge": ([P, P, P, P, P, I64, I32, I32, I32, P], I32),
    "dan_quantize_e4m3_tensor": ([P, I64, P, I64, P, I32, I32, P], I32),
}

_lib = None


def lib():
    """The loaded library (loaded on first use)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m dan_b200.build` "
                               "(dan_b200 has no CPU fallback)")
        lb = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lb, name, None)
            if fn is None:
                continue
            fn.argtypes, fn.restype = args, res
        _lib = lb
    return _lib


def exported():
    """Names of the C-ABI symbols the library exports (of those this binding knows)."""
    lb = lib()
    return [n for n in SIGNATURES if hasattr(lb, n)]


def call(name, *args, work=0, key=None):
    """Launch entry point ``name``; ``work`` is its algorithmic FLOPs or bytes, ``key`` the
    group its timing is reported under (default: the entry point)."""
    fn = getattr(lib(), name)
    timer = profiling.active()
    if timer is not None and timer.wants(name):
        s, e = timer.event(), timer.event()
        s.record()
        rc = fn(*args)
        e.record()
        timer.records[key or name].append((s, e, work))
    else:
        rc = fn(*args)
    if rc != 0:
        raise RuntimeError(f"{name}: {lib().dan_last_error().decode()} (code {rc})")
    profiling.launches[name] += 1


def delta_scratch(n_chunks, hk, hv, device):
    """Scratch tensor for dan_gated_delta_scan (reused across the layers of one forward)."""
    return torch.empty(max(int(lib().dan_gated_delta_scratch_bytes(n_chunks, hk, hv)), 16), dtype=torch.uint8,
                       device=device)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


_status = {}


def status_word(device):
    """The per-device int32 status word kernels report bounded-wait timeouts and bad indices into."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    s = _status.get(idx)
    if s is None:
        # a normal tensor even when the first caller runs under torch.inference_mode (as
        # Runner.read_many does): check_status clears it in place from any mode
        with torch.inference_mode(False):
            s = _status[idx] = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
    return s


STATUS_TEXT = {1: "a TMA load never landed", 2: "a pipeline stage was never released",
               3: "an MMA commit never arrived", 4: "the softmax warps never finished", 5: "an index was out of range",
               6: "a stream-K partial tile never arrived"}


def check_status(device):
    """Raise if any kernel on ``device`` reported an error since the last check (synchronises)."""
    s = status_word(device)
    v = int(s.item())
    if v:
        s.zero_()
        raise RuntimeError(f"dan_b200 kernel error {v}: {STATUS_TEXT.get(v, 'unknown')}")
