"""The planner's template cache (dan_b200.planner.CachedPlanner) against dan's own Planner
(dan/prompt.py:70-227) on a synthetic byte-level BPE tokenizer with a chat template (no model
download): identical read plans over random states, question sets, option rotations, both
layouts and both label styles, with far fewer renders of the chat template. A template that
trims its content cannot be framed; the cache then keeps dan's path and plans stay identical."""
import random
import string
import types

import pytest

pytest.importorskip("dan.prompt")

from dan.prompt import Planner  # noqa: E402

from dan_b200.planner import CachedPlanner  # noqa: E402

VERBATIM = ("{{ bos_token }}{% for m in messages %}<|start|>{{ m['role'] }}<|end|>\n\n{{ m['content'] }}<|eot|>"
            "{% endfor %}{% if add_generation_prompt %}<|start|>assistant<|end|>\n\n{% endif %}")
TRIMMING = VERBATIM.replace("{{ m['content'] }}", "{{ m['content'] | trim }}")


def _tokenizer(template, seed=0):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
    from transformers import PreTrainedTokenizerFast

    rng = random.Random(seed)
    words = ["".join(rng.choice(string.ascii_lowercase) for _ in range(rng.randint(2, 8))) for _ in range(300)]
    corpus = [" ".join(rng.choice(words) for _ in range(30)) for _ in range(400)]
    corpus += list(string.ascii_letters) + list(string.digits) + ["yes no Yes No Y N A B", "Reply with the label only."]
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    specials = ["<|begin|>", "<|start|>", "<|end|>", "<|eot|>"]
    tok.train_from_iterator(corpus, trainers.BpeTrainer(vocab_size=900, special_tokens=specials,
                                                        initial_alphabet=pre_tokenizers.ByteLevel.alphabet()))
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, bos_token="<|begin|>", eos_token="<|eot|>")
    fast.chat_template = template
    return fast, words


def _questions(rng, words):
    qs = {}
    for i in range(rng.randint(1, 4)):
        kind = rng.choice(["noul", "choice", "score"])
        q = {"type": kind, "instructions": " ".join(rng.choice(words) for _ in range(rng.randint(2, 9))) + "?"}
        if kind == "choice":
            q["criteria"] = {rng.choice(words) + str(j): rng.choice([None, rng.choice(words)])
                             for j in range(rng.randint(2, 6))}
        elif kind == "score":
            q["criteria"] = [rng.choice(words) for _ in range(rng.randint(2, 5))]
        qs[f"q{i}_{kind}"] = q
    return qs


def _state(rng, words):
    text = " ".join(rng.choice(words) for _ in range(rng.randint(5, 120)))
    if rng.random() < 0.3:
        text = rng.choice([" ", "\n", "  \n"]) + text + rng.choice([" ", "\n\n", ""])
    if rng.random() < 0.3:
        return {"message": text, "n": rng.randint(0, 99)}
    return text


@pytest.mark.parametrize("template,framed", [(VERBATIM, True), (TRIMMING, False)])
def test_cached_planner_matches_dan(template, framed):
    tok, words = _tokenizer(template)
    rng = random.Random(1)
    ref, cached = Planner(tok), CachedPlanner(tok)
    for _ in range(40):
        state, qs = _state(rng, words), _questions(rng, words)
        profile = types.SimpleNamespace(label_style=rng.choice(["letters", "names"]),
                                        layout=rng.choice(["inline", "system"]), permutations=rng.randint(1, 3))
        assert cached.plans(state, qs, profile) == ref.plans(state, qs, profile)
    assert (cached.frame(None) is not None) == framed
    if framed:  # the template is rendered for its frame probes only, not per prompt
        assert cached.template_calls * 10 < ref_calls(ref, tok, words)


def ref_calls(ref, tok, words):
    """Template renders dan's planner makes for the same workload."""
    calls = 0
    original = ref.render

    def counting(system, user, tokenize):
        nonlocal calls
        calls += 1
        return original(system, user, tokenize)

    ref.render = counting
    rng = random.Random(1)
    for _ in range(40):
        state, qs = _state(rng, words), _questions(rng, words)
        profile = types.SimpleNamespace(label_style=rng.choice(["letters", "names"]),
                                        layout=rng.choice(["inline", "system"]), permutations=rng.randint(1, 3))
        ref.plans(state, qs, profile)
    return calls


def test_prompt_ids_cache_is_bounded():
    tok, words = _tokenizer(VERBATIM)
    cached = CachedPlanner(tok, memo=8)
    for i in range(50):
        cached.prefix_ids(None, f"state {i}")
    assert len(cached._ids) == 8
    assert cached.prefix_ids(None, "state 49") == Planner(tok).prefix_ids(None, "state 49")
