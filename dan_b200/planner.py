"""Prompt planning with the chat template rendered once, not per prompt (dan/prompt.py:70-123,
202-227).

dan's ``Planner`` renders the model's chat template (Jinja) and tokenizes the whole prompt for
every call of ``prefix_ids`` / ``prompt_text``: per read plan at least the state with its first
question and the same state with a probe question, and each option rotation of a request
(``profile.permutations``) plans the whole request again. Once the GPU path reads a batch in a
few milliseconds, this host work is what limits answers per second.

``CachedPlanner`` is dan's planner with two caches and nothing else changed:

- the template's *frame*, learnt once for prompts without and once for prompts with a system
  message: the rendered text around the contents, from a few probe renders, accepted only if the
  template inserts the contents verbatim (probes with surrounding whitespace and newlines must
  survive untouched) and if tokenizing the framed text gives exactly the ids
  ``apply_chat_template(tokenize=True)`` gives. A prompt is then a string concatenation and one
  tokenizer call, whatever the schema; a template that rewrites its contents (trims them, say)
  keeps dan's path;
- the token ids of recent ``(system, user)`` prompts (bounded LRU), which the probe prompt of
  every rotation after the first and every request repeating a state hit.

Plans are identical to dan's (``tests/test_planner.py`` compares them over random states,
question sets, rotations, layouts and label styles on a synthetic tokenizer). dan's planner is
dan's own code, installed beside this package.
"""
import threading
from collections import OrderedDict

from . import _dan

MARK_A = "@@dan-b200-frame-a@@"
MARK_B = "@@dan-b200-frame-b@@"


def _base():
    return _dan._need("dan.prompt").Planner


def CachedPlanner(tokenizer, memo=512):  # noqa: N802 - a class factory named like the class it returns
    """dan's ``Planner`` over ``tokenizer`` with the template frame and prompt-ids caches."""
    return _cached_class()(tokenizer, memo)


_CLASS = None


def _cached_class():
    global _CLASS
    if _CLASS is not None:
        return _CLASS
    base = _base()

    class _CachedPlanner(base):
        def __init__(self, tokenizer, memo=512):
            super().__init__(tokenizer)
            self._frames = {}
            self._ids = OrderedDict()
            self._memo = memo
            self._lock = threading.Lock()  # the engine plans on a thread pool
            self.template_calls = 0  # renders of the real chat template (statistics)

        def render(self, system, user, tokenize):
            self.template_calls += 1
            return super().render(system, user, tokenize)

        def _real_ids(self, system, user):
            return base.prefix_ids(self, system, user)

        def _frame(self, with_system):
            """The template around its content, learnt once: (before, after) with
            render(None, u) == before + u + after, or (before, mid, after) with
            render(s, u) == before + s + mid + u + after; None when the template does not insert
            its content verbatim or tokenizing the framed text differs from its own tokenization."""
            if with_system in self._frames:
                return self._frames[with_system]
            f = None
            pad_a, pad_b = " \n" + MARK_A + "\n\n ", "\n" + MARK_B + "  "
            if not with_system:
                a = base.prompt_text(self, None, MARK_A)
                i = a.find(MARK_A)
                if i >= 0 and a.count(MARK_A) == 1:
                    cand = (a[:i], a[i + len(MARK_A):])
                    if all(base.prompt_text(self, None, u) == cand[0] + u + cand[1] for u in (MARK_B, pad_a, pad_b)):
                        f = cand
            else:
                a = base.prompt_text(self, MARK_B, MARK_A)
                if self._supports_system:  # the template has a system role: both contents are framed
                    i, j = a.find(MARK_B), a.find(MARK_A)
                    if 0 <= i < j and a.count(MARK_A) == 1 and a.count(MARK_B) == 1:
                        cand = (a[:i], a[i + len(MARK_B):j], a[j + len(MARK_A):])
                        if all(base.prompt_text(self, s_, u) == cand[0] + s_ + cand[1] + u + cand[2]
                               for s_, u in ((pad_b, pad_a), (MARK_A, MARK_B))):
                            f = cand
            if f is not None:  # the framed text must tokenize exactly as the template's own call does
                s_, u = ("x " + MARK_B + "\n", "y\n\n" + MARK_A + " z") if with_system else (None, "x " + MARK_A + "\n\ny")
                text = self._join(f, s_, u)
                if [int(t) for t in self.tok.encode(text, add_special_tokens=False)] != self._real_ids(s_, u):
                    f = None
            self._frames[with_system] = f
            return f

        @staticmethod
        def _join(f, system, user):
            return f[0] + user + f[1] if len(f) == 2 else f[0] + system + f[1] + user + f[2]

        def frame(self, system):
            """The frame that applies to prompts with (or without) a system text, or None."""
            if system is not None and self._supports_system is False:
                return None  # dan folds the system text into the user message: its own path
            return self._frame(system is not None)

        def prompt_text(self, system, user):
            f = self.frame(system)
            if f is None:
                return base.prompt_text(self, system, user)
            return self._join(f, system, user)

        def prefix_ids(self, system, user):
            key = (system, user)
            with self._lock:
                hit = self._ids.get(key)
                if hit is not None:
                    self._ids.move_to_end(key)
                    return list(hit)
            f = self.frame(system)
            if f is None:
                ids = self._real_ids(system, user)
            else:
                ids = [int(t) for t in self.tok.encode(self._join(f, system, user), add_special_tokens=False)]
            with self._lock:
                self._ids[key] = tuple(ids)
                if len(self._ids) > self._memo:
                    self._ids.popitem(last=False)
            return ids

    _CLASS = _CachedPlanner
    return _CLASS
