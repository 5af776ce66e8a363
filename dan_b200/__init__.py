"""dan on B200: the packed prefill read path of dan, as hand-written sm_100a CUDA.

The host side mirrors dan's own interfaces (``Runner``, ``LLM``,
``AsyncEngine``, the model classes' ``hidden`` / ``label_logits``); the
compute runs in ``libdan_b200.so``, a C-ABI library of tcgen05 / TMA kernels
declared in ``include/dan_b200.h``.
"""
__version__ = "0.1.0"
