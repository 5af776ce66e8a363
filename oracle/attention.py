"""Tree-masked attention, restated on the CPU (test infrastructure only).

Follows dan/attention.py of the reference:

- the visibility rule "key comes first and (key is trunk or same branch)"
  (attention.py:6-13, ``tree_mask`` 54-59, ``branch_rows_mask`` 62-69);
- cached ``past`` keys are trunk, visible to every query of the segment
  (attention.py:12-13, ``Segment.mask`` 86-95);
- the dense reference computation ``_attend_dense`` (attention.py:244-270):
  per segment, softmax(q k^T * scale) v over ``[past; new]`` keys with GQA head
  sharing (query head h reads kv head h // (H / Hkv), attention.py:273-279).

The computation here is an explicit masked softmax in fp64, so it serves as
the exact answer for both the trunk-causal and the branch rows.
"""
import torch


def tree_mask(branch):
    """[N, N] bool (True = attend) from per-token branch ids, 0 = trunk (attention.py:54-59)."""
    n = branch.shape[0]
    idx = torch.arange(n)
    causal = idx[None, :] <= idx[:, None]
    return causal & ((branch[None, :] == 0) | (branch[None, :] == branch[:, None]))


def branch_rows_mask(branch, trunk):
    """Rows ``trunk:`` of ``tree_mask(branch)`` (attention.py:62-69)."""
    return tree_mask(branch)[trunk:]


def segment_mask(branch_ids, past_len):
    """Visibility of one segment: rows = its new tokens, cols = [past; new] (attention.py:86-95, 258-269)."""
    m = tree_mask(torch.as_tensor(branch_ids, dtype=torch.long))
    if past_len:
        m = torch.cat([torch.ones(m.shape[0], past_len, dtype=torch.bool), m], dim=1)
    return m


def attend(q, k, v, segments, scale=None, p_bf16=False):
    """q: [H, N, D]; k, v: [Hkv, N, D] -> [H, N, D] (fp32).

    ``segments``: list of dicts ``{"start", "end", "branch": [ids per new token],
    "past": None or (pk, pv) each [Hkv, past, D]}``. ``p_bf16``: the unnormalised
    probabilities exp(s - rowmax) rounded to bf16 before they multiply V (normalised by their
    unrounded sum), as a tensor-core attention kernel feeds them to its PV product; used to
    measure how far that rounding alone moves a model's answers."""
    h, n, d = q.shape
    rep = h // k.shape[0]
    scale = d ** -0.5 if scale is None else scale
    out = torch.zeros(h, n, d, dtype=torch.float32)
    for s in segments:
        a, b = s["start"], s["end"]
        ks, vs = k[:, a:b].double(), v[:, a:b].double()
        past = 0
        if s.get("past") is not None:
            pk, pv = s["past"]
            past = pk.shape[1]
            ks, vs = torch.cat([pk.double(), ks], 1), torch.cat([pv.double(), vs], 1)
        mask = segment_mask(s["branch"], past)
        ks = ks.repeat_interleave(rep, 0)
        vs = vs.repeat_interleave(rep, 0)
        sc = (q[:, a:b].double() @ ks.transpose(1, 2)) * scale
        sc = sc.masked_fill(~mask[None], float("-inf"))
        if p_bf16:
            e = torch.exp(sc - sc.amax(-1, keepdim=True))
            out[:, a:b] = ((e.float().bfloat16().double() @ vs) / e.sum(-1, keepdim=True)).float()
        else:
            out[:, a:b] = (torch.softmax(sc, -1) @ vs).float()
    return out


def useful_pairs(segments):
    """Visible (query, key) pairs of a packed batch: the attention work unit.

    Per segment with t new trunk tokens, past P and branches of length l_b:
    t(t+1)/2 + P*t + sum_b (l_b (P + t) + l_b (l_b + 1) / 2)."""
    total = 0
    for s in segments:
        br = list(s["branch"])
        t = next((i for i, x in enumerate(br) if x), len(br))
        p = 0 if s.get("past") is None else s["past"][0].shape[1]
        total += t * (t + 1) // 2 + p * t
        i = t
        while i < len(br):
            j = i
            while j < len(br) and br[j] == br[i]:
                j += 1
            length = j - i
            total += length * (p + t) + length * (length + 1) // 2
            i = j
    return total
