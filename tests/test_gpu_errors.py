"""Error paths on the GPU, in the forms that leave the device usable (no fault, no hang):

- an out-of-range token id or label id is a bounds-checked read: the kernel records
  kBadIndex in the status word, and ``read_many`` raises ``RuntimeError`` for that batch (dan's
  engine then fails only that batch, dan/engine.py:102-107); the next batch reads normally;
- a bounded wait that runs out (an mbarrier phase or a device flag that nothing completes)
  reports its timeout code and the kernel returns;
- bad arguments are refused on the host before any launch with a negative code, raised as
  ``RuntimeError`` with the library's text."""
import ctypes

import pytest
import torch

from dan_b200 import _lib, ops
from dan_b200.plan import Branch, ReadPlan
from dan_b200.runner import Runner
from oracle import weights

pytestmark = pytest.mark.gpu

VOCAB = 512


@pytest.fixture(scope="module")
def runner(cuda, tmp_path_factory):
    cfg = weights.llama_config(vocab=VOCAB, hidden=256, inter=512, layers=2, heads=4, kv_heads=2, head_dim=64)
    path = tmp_path_factory.mktemp("tiny_errors")
    weights.save_checkpoint(str(path), cfg, weights.random_state(cfg, seed=3))
    return Runner(str(path), cuda, cache_bytes=0)


GOOD = [ReadPlan(list(range(10, 90)), branches=[Branch([7, 8], [1, 2, 3])])]


def test_bad_token_id_fails_the_batch_only(runner):
    want = runner.read_many(GOOD)
    bad = [ReadPlan(list(range(10, 90)) + [VOCAB + 5], branches=[Branch([7, 8], [1, 2, 3])])]
    with pytest.raises(RuntimeError, match="index was out of range"):
        runner.read_many(bad)
    again = runner.read_many(GOOD)  # the status word was cleared; the device still works
    assert torch.equal(again[0][0], want[0][0])


def test_bad_label_id_fails_the_batch_only(runner):
    bad = [ReadPlan(list(range(10, 90)), branches=[Branch([7, 8], [1, VOCAB])])]
    with pytest.raises(RuntimeError, match="index was out of range"):
        runner.read_many(bad)
    runner.read_many(GOOD)


def test_readout_more_labels_than_slots(cuda):
    h = torch.randn(4, 256, device=cuda).bfloat16()
    table = torch.randn(VOCAB, 256, device=cuda).bfloat16()
    nw = torch.ones(256, device=cuda).bfloat16()
    rows = torch.tensor([0, 3], dtype=torch.int32, device=cuda)
    labels = torch.arange(9, dtype=torch.int32, device=cuda)
    off = torch.tensor([0, 3, 9], dtype=torch.int32, device=cuda)  # the second question has 6 labels
    ops.label_readout(h, rows, nw, 1e-5, ops.NORM_LLAMA, table, labels, off, 4)  # room for 4
    with pytest.raises(RuntimeError, match="index was out of range"):
        _lib.check_status(cuda)
    lg, _ = ops.label_readout(h, rows, nw, 1e-5, ops.NORM_LLAMA, table, labels, off, 6)
    _lib.check_status(cuda)
    assert torch.isfinite(lg).all()


@pytest.mark.parametrize("kind,code", [(0, 1), (1, 6)])
def test_bounded_wait_reports_timeout(cuda, kind, code):
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.call("dan_selftest_wait", kind, _lib.ptr(flag), _lib.ptr(status), _lib.stream())
    torch.cuda.synchronize()
    assert int(status.item()) == code
    assert _lib.STATUS_TEXT[code]
    x = torch.randn(256, 256, device=cuda).bfloat16()  # the context is still usable
    torch.testing.assert_close(ops.linear(x, x).float(), x.float() @ x.float().T, atol=0.5, rtol=2e-2)


def test_bad_arguments_raise(cuda):
    x = torch.randn(256, 512, device=cuda).bfloat16()
    w = torch.randn(384, 512, device=cuda).bfloat16()
    out = torch.empty(256, 384, device=cuda, dtype=torch.bfloat16)
    st = _lib.ptr(_lib.status_word(cuda))
    with pytest.raises(RuntimeError, match="16-byte"):  # lda of 511 elements: rows not 16-byte aligned
        _lib.call("dan_gemm_bf16", _lib.ptr(x), 511, _lib.ptr(w), 512, _lib.ptr(out), 384, None, 0, None, 256, 384,
                  511, 0, st, _lib.stream())
    with pytest.raises(RuntimeError, match="unknown epilogue"):
        _lib.call("dan_gemm_bf16", _lib.ptr(x), 512, _lib.ptr(w), 512, _lib.ptr(out), 384, None, 0, None, 256, 384,
                  512, 7, st, _lib.stream())
    with pytest.raises(RuntimeError, match="head_dim 96 unsupported"):
        _lib.call("dan_tree_attention", _lib.ptr(x), 512, 96, _lib.ptr(x), 512, 96, _lib.ptr(x), 512, 96, None,
                  None, 0, 0, 0, _lib.ptr(out), 384, 96, 256, 4, 2, 96, None, 1, None, None, None, 0,
                  ctypes.c_float(0.1), st, _lib.stream())
    assert _lib.lib().dan_gemm_bf16(None, 0, None, 0, None, 0, None, 0, None, 0, 8, 8, 0, None, None) == -22
