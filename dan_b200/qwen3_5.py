"""Qwen3.5 hybrid (Gated DeltaNet + gated attention) on the dan_b200 kernels."""


class Qwen35ForReads:
    MODEL_TYPES = frozenset({"qwen3_5", "qwen3_5_text"})

    def __init__(self, *args, **kwargs):
        raise NotImplementedError("the Qwen3.5 DeltaNet kernels are not built yet")
