"""dan_gemm_bf16_noalloc against dan_gemm_bf16 (collected last, after every other GPU test).

The allocation-free entry point keeps the stream-K partial tiles in the library's static
device scratch instead of a cudaMalloc'd workspace. On the same inputs it must return exactly
what dan_gemm_bf16 returns, on a first and a second call (the second reuses the scratch and
its per-launch epoch), for shapes that take the stream-K path and one that does not."""
import pytest
import torch

from dan_b200 import _lib

pytestmark = pytest.mark.gpu

STORE, RESIDUAL = 0, 1


def _gemm(name, x, w, out, resid, ep):
    m, k = x.shape
    n = w.shape[0]
    _lib.call(name, _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(out), out.stride(0),
              _lib.ptr(resid), resid.stride(0) if resid is not None else 0, None, m, n, k, ep,
              _lib.ptr(_lib.status_word(x.device)), _lib.stream())


# (7089, 4096, 14336) and (300, 1024, 8192) take stream-K; (1000, 768, 512) does not.
@pytest.mark.parametrize("m,n,k", [(7089, 4096, 14336), (300, 1024, 8192), (1000, 768, 512)])
@pytest.mark.parametrize("ep", [STORE, RESIDUAL])
def test_noalloc_matches_allocating_entry(cuda, m, n, k, ep):
    g = torch.Generator(device=cuda).manual_seed(m + n + k + ep)
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.05).bfloat16()
    r = torch.randn(m, n, device=cuda, generator=g).bfloat16() if ep == RESIDUAL else None
    for call in range(2):
        want = r.clone() if r is not None else torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
        got = r.clone() if r is not None else torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
        _gemm("dan_gemm_bf16", x, w, want, want if r is not None else None, ep)
        _gemm("dan_gemm_bf16_noalloc", x, w, got, got if r is not None else None, ep)
        torch.cuda.synchronize()
        _lib.check_status(cuda)
        assert torch.equal(got, want), f"call {call}: noalloc differs from dan_gemm_bf16"
