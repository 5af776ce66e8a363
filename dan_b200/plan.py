"""Read plans: the input contract of the packed prefill path.

Same field names and meaning as the reference planner's output
(dan/prompt.py:31-47): a shared ``prefix`` (the trunk prompt), one ``Branch``
per question (its ``suffix`` tokens, read at the last one, over ``label_ids``),
and ``static``, the number of leading prefix tokens that are cacheable. The
tokenizer-bound planner itself is outside this package; any object with these
attributes is accepted by the runner.
"""
from dataclasses import dataclass, field


@dataclass
class Branch:
    suffix: list  # tokens after the shared prefix; the last one is the read position
    label_ids: list  # one token per option, in option order


@dataclass
class ReadPlan:
    prefix: list
    specs: list = field(default_factory=list)
    labels: list = field(default_factory=list)
    branches: list = field(default_factory=list)
    forced: dict = field(default_factory=dict)
    order: list = field(default_factory=list)
    static: int = 0
    perms: list = field(default_factory=list)
