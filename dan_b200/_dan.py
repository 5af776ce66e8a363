"""dan's own host code that this package calls but does not rebuild.

Answer formatting (label log-probabilities in canonical option order, the
average over option rotations, Jev answer dicts: dan/readout.py:13-68) and the
prompt planner (dan/prompt.py) stay dan's code: they do no device work. dan is
installed beside this package (``pip install`` of the reference, or its
source tree on ``sys.path``); this module imports it on first use and says
so clearly when it is missing.
"""


def _need(name):
    import importlib

    try:
        return importlib.import_module(name)
    except ImportError as e:  # pragma: no cover - depends on the environment
        raise ImportError(f"{name} is dan's own code and must be installed beside dan_b200 "
                          f"(pip install the reference package): {e}") from e


def answers(plan, label_logits, profile=None, logits_canonical=False):
    """dan.readout.answers (dan/readout.py:59-68)."""
    return _need("dan.readout").answers(plan, label_logits, profile, logits_canonical=logits_canonical)


def combine(plans, reads):
    """dan.readout.combine (dan/readout.py:52-56)."""
    return _need("dan.readout").combine(plans, reads)


def planner(tokenizer):
    """dan.prompt.Planner over ``tokenizer`` (dan/prompt.py:70-123)."""
    return _need("dan.prompt").Planner(tokenizer)
