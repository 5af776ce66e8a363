"""CPU oracle for dan's packed prefill read path — TEST INFRASTRUCTURE ONLY.

This package restates, in plain fp32 PyTorch on the CPU, the algorithm of the
reference project (quangliz/dan) for the hot path that ``dan_b200`` rebuilds on
B200: tree-masked attention, the Llama and Qwen3.5 decoders, the gated delta
rule, FP8 per-token / per-channel quantisation and the label readout. Every
function cites the reference ``file:line`` it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline
leg may import it, and only as the checker (or the timed CPU arm), never as
the thing measured or shipped: the ``dan_b200`` product path never imports
this package and fails loudly when its CUDA library is missing.

Pinning: the attention, Llama, Qwen3.5 and packing restatements are checked
against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``). The reference's FP8 path needs a CUDA GPU
and has no test of its own, so no fixture pins the FP8 restatement here; on
the GPU box, ``tests/test_gpu_model.py`` runs the reference's own FP8 path
(its offline install) and checks this restatement against it (3e-2 on
probabilities).
"""
