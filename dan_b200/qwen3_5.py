"""Qwen3.5 hybrid (Gated DeltaNet + gated attention), text only, prefill only, on the
dan_b200 kernels.

Same interface and numerics as the reference's ``Qwen35ForReads``
(dan/models/qwen3_5.py:375-420): three of every four layers are Gated DeltaNet,
the rest gated attention with q/k zero-centred RMSNorm, partial RoPE and a
per-head sigmoid output gate; norms are zero-centred (x_hat * (1 + w)).

Per DeltaNet layer on the GPU (qwen3_5.py:183-212): merged in_proj GEMM ->
causal depthwise conv + SiLU over each run's ``[history; tokens]``
(``dan_causal_conv``, history from a per-row index table) -> gated delta scan
over the tree of runs with gates, l2-norms and q scaling fused
(``dan_gated_delta_scan``; branches fork from the trunk's final state kept on
chip) -> gated RMSNorm -> out_proj GEMM with the residual add fused. Prefix
saves store the state at the save cut and the conv tail into the pool's slot.

Per attention layer (qwen3_5.py:316-329): merged q/k/v GEMM -> per-head q/k
norms in place -> partial RoPE in place -> tree attention reading the strided
q (head stride 2d, the gate interleaved) -> sigmoid gate in place -> o GEMM +
residual. The MLP matches the Llama path (SwiGLU fused into the gate/up GEMM).
"""
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, ops
from .attention import layout_of, tree_attention
from .llama import Linear, _label_logits

PRE = "model.language_model."


def remap(name):
    """Checkpoint key -> this module's key, or None to skip (vision, MTP) (qwen3_5.py:394-401)."""
    if name.startswith(PRE):
        return "model." + name[len(PRE):]
    if name.startswith("model.") and not name.startswith("model.visual"):
        return name
    if name.startswith("lm_head."):
        return name
    return None


CHUNK = 64  # tokens per chunk of the scan


def delta_rule(q, k, v, g, beta, lengths, states, cu=None):
    """Gated delta rule over packed sequences of ``lengths`` (qwen3_5.py:136-158): q, k [N, H,
    128], v [N, H, 128] bf16 (q and k are l2-normalised and q scaled by 128^-0.5 inside, as
    dan's kernels do), g [N, H] fp32 log decay, beta [N, H] bf16, ``states`` [S, H, 128, 128]
    fp32 initial states, one per sequence. Returns (out [N, H, 128] bf16, final states fp32).
    ``cu`` (dan's precomputed cumulative lengths) is accepted and not needed: each sequence is
    one run of 64-token chunks of the chunked scan, its final state stored in place of a copy
    of its initial one."""
    n, h, dk = q.shape
    dv = v.shape[-1]
    lengths = [int(x) for x in lengths]
    if sum(lengths) != n or len(lengths) != states.shape[0]:
        raise ValueError(f"delta_rule: lengths {sum(lengths)} / {len(lengths)} do not match {n} rows / "
                         f"{states.shape[0]} states")
    for t in (q, k, v, beta):
        if not (t.is_cuda and t.dtype == torch.bfloat16):
            raise ValueError("delta_rule: q, k, v and beta must be bf16 CUDA tensors")
    dev = q.device
    final = states.to(torch.float32).contiguous().clone()
    segs, chunks, start = [], [], 0
    for i, length in enumerate(lengths):
        segs.append((start, length, length, i, i, 0, 0, len(chunks)))
        chunks += [(start + t0, min(CHUNK, length - t0)) for t0 in range(0, length, CHUNK)]
        start += length
    segs.sort(key=lambda r: -r[1])
    up = lambda a, cols: torch.as_tensor(np.asarray(a, dtype=np.int32).reshape(-1, cols)).to(dev)  # noqa: E731
    segs_t, chunks_t, br_t = up(segs, 8), up(chunks or [(0, 0)], 2), up([(0, 0, 0, 0)], 4)
    qkv = torch.cat([q.reshape(n, -1), k.reshape(n, -1), v.reshape(n, -1)], 1)  # one row stride for all three
    beta2 = beta.reshape(n, h).contiguous()
    g2 = g.reshape(n, h).to(torch.float32).contiguous()
    out = torch.empty(n, h, dv, dtype=torch.bfloat16, device=dev)
    scratch = _lib.delta_scratch(len(chunks), h, h, dev)
    kd = h * dk
    _lib.call("dan_delta_rule_scan", _lib.ptr(qkv), _lib.ptr(qkv[:, kd:]), _lib.ptr(qkv[:, 2 * kd:]), qkv.stride(0),
              _lib.ptr(beta2), beta2.stride(0), _lib.ptr(g2), g2.stride(0), _lib.ptr(segs_t), len(segs),
              _lib.ptr(br_t), _lib.ptr(chunks_t), len(chunks), _lib.ptr(final), final.stride(0), _lib.ptr(out),
              h * dv, h, h, dk, dv, float(dk ** -0.5), _lib.ptr(scratch), scratch.numel(),
              _lib.ptr(_lib.status_word(dev)), _lib.stream())
    return out, final


@dataclass
class RecurrentLayout:
    """Index tables of one batch for the DeltaNet layers (the reference's RecurrentLayout,
    qwen3_5.py:240-298, as per-row conv sources, per-segment scan records and the chunk list).

    A segment's runs are its trunk up to the save cut, the rest of the trunk and each
    branch; every run is cut into chunks of ``CHUNK`` rows, listed contiguously per segment in
    processing order. Segment records are sorted longest first (the scan's CTAs for the
    longest chains start first)."""
    prev: torch.Tensor  # int32 [N, 3]: conv source codes of the 1st/2nd/3rd previous rows
    segs: torch.Tensor  # int32 [S, 8]: trunk_start, trunk_len, cut, init_slot, save_slot, branch0, n_br, chunk0
    branches: torch.Tensor  # int32 [B, 4]: start, len, chunk0, 0
    chunks: torch.Tensor  # int32 [C, 2]: first row, rows (<= CHUNK)
    tail_codes: torch.Tensor  # int32 [saves * (k-1)]: conv-tail source codes at each save cut
    tail_dst: list  # (slot) per save
    n_segs: int
    n_rows: int
    n_chunks: int = 0
    n_state_io: int = 0  # fp32 states the scan reads (cached pasts) plus writes (save cuts)
    lead: tuple = (0, 0)  # (first chunk, chunks) of segment 0 when the scan should split, else (0, 0)

    # The scan's split launch (segment 0's chain beside the other segments' pre-pass) pays when
    # that chain outlasts the rest of the pre-pass: measured on B200 at 128-wide heads, a chain
    # takes ~2.3 us per chunk and the pre-pass ~0.054 us per chunk and value head, slowed by
    # ~30% while it shares the GPU with the chain. So split when the leading segment has at
    # least MIN_LEAD chunks and leads the next one by more than the share of the rest of the
    # pre-pass the overlap costs.
    MIN_LEAD = 8

    @staticmethod
    def split_lead(counts, hv):
        """counts: chunks per segment, longest segment first. (index of its first chunk is the
        caller's) -> whether the scan should split off segment 0."""
        if len(counts) < 2 or counts[0] < RecurrentLayout.MIN_LEAD:
            return False
        rest = sum(counts) - counts[0]
        return 2.3 * (counts[0] - max(counts[1:])) > 0.3 * 0.054 * hv * rest

    @classmethod
    def build(cls, segments, n_rows, k1, device):
        prev = np.full((max(n_rows, 1), k1), -1, dtype=np.int32)
        segs, brs, tail, tail_dst, chunks = [], [], [], [], []

        def cut_runs(start, length):
            first = len(chunks)
            for t0 in range(0, length, CHUNK):
                chunks.append((start + t0, min(CHUNK, length - t0)))
            return first

        for s in segments:
            slot = s.past.slot if s.past else -1
            hist = [-(2 + slot * k1 + j) for j in range(k1)] if s.past else [-1] * k1
            virt = hist + list(range(s.start, s.start + s.trunk))
            for t in range(s.trunk):
                for j in range(k1):
                    prev[s.start + t, j] = virt[k1 + t - 1 - j]
            tail_hist = virt[-k1:]
            for a, b in s.branches:
                bv = tail_hist + list(range(a, b))
                for t in range(b - a):
                    for j in range(k1):
                        prev[a + t, j] = bv[k1 + t - 1 - j]
            cut = s.save if 0 < s.save < s.trunk else s.trunk
            save_slot = s.save_entry.slot if getattr(s, "save_entry", None) is not None else -1
            if save_slot >= 0:
                tail += virt[cut:k1 + cut]
                tail_dst.append(save_slot)
            chunk0 = cut_runs(s.start, cut)
            cut_runs(s.start + cut, s.trunk - cut)
            b0 = len(brs)
            for a, b in s.branches:
                brs.append((a, b - a, cut_runs(a, b - a), 0))
            # the record, then (not uploaded) its chunk count: a segment's chunks are contiguous
            segs.append((s.start, s.trunk, cut, slot, save_slot, b0, len(s.branches), chunk0, len(chunks) - chunk0))
        segs.sort(key=lambda r: -(r[1] + sum(brs[r[5] + i][1] for i in range(r[6]))))
        seg_chunks = [(r[7], r[8]) for r in segs]  # (first chunk, chunks), longest segment first
        segs = [r[:8] for r in segs]
        dev = torch.device(device)

        def up(a, shape):
            t = torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.int32).reshape(shape)))
            return t.pin_memory().to(dev, non_blocking=True) if dev.type == "cuda" else t

        io = sum((r[3] >= 0) + (r[4] >= 0) for r in segs)
        lay = cls(up(prev[:max(n_rows, 1)], (-1, k1)), up(segs, (-1, 8)), up(brs or [(0, 0, 0, 0)], (-1, 4)),
                  up(chunks or [(0, 0)], (-1, 2)), up(tail or [0], (-1,)), tail_dst, len(segs), n_rows,
                  len(chunks), int(io))
        lay.seg_chunks = seg_chunks
        return lay

    def choose_lead(self, hv):
        """Set ``lead`` for a layer with ``hv`` value heads (``split_lead``'s rule)."""
        counts = [c for _, c in self.seg_chunks]
        self.lead = self.seg_chunks[0] if self.split_lead(counts, hv) else (0, 0)
        return self.lead


class Qwen35ForReads:
    MODEL_TYPES = frozenset({"qwen3_5", "qwen3_5_text"})

    def __init__(self, config, state, device="cuda", dtype=torch.bfloat16, quantization=None):
        if dtype != torch.bfloat16:
            raise ValueError("dan_b200 runs the decoder in bf16")
        if quantization:
            raise ValueError("FP8 is supported for the Llama family only")
        c = self.config = dict(config.get("text_config", config))
        self.device = torch.device(device)
        st = {}
        for k, v in state.items():
            k2 = remap(k)
            if k2 is not None:
                st[k2] = v
        self.h, self.hkv, self.d = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        self.hk, self.hv = c["linear_num_key_heads"], c["linear_num_value_heads"]
        self.dk, self.dv = c["linear_key_head_dim"], c["linear_value_head_dim"]
        self.kconv = c["linear_conv_kernel_dim"]
        self.conv_dim = 2 * self.hk * self.dk + self.hv * self.dv
        self.eps = c["rms_norm_eps"]
        self.kinds = list(c["layer_types"])
        rp = c.get("rope_parameters") or {"rope_theta": c.get("rope_theta", 10000.0)}
        self.rot = int(self.d * rp.get("partial_rotary_factor", 1.0))

        def g(name):
            return st[name].to(self.device, torch.bfloat16)

        def g32(name):  # stored in the model dtype, used in fp32 (qwen3_5.py:188, fused.py:79-82)
            return st[name].to(self.device, torch.bfloat16).float()

        self.embed_tokens = g("model.embed_tokens.weight").contiguous()
        self.lm_head = g("lm_head.weight").contiguous() if "lm_head.weight" in st else self.embed_tokens
        self.norm = g("model.norm.weight")
        self.layers = []
        self.attn_index, self.delta_index = {}, {}
        for i, kind in enumerate(self.kinds):
            p = f"model.layers.{i}."
            L = {"kind": kind, "in_norm": g(p + "input_layernorm.weight"),
                 "post_norm": g(p + "post_attention_layernorm.weight"),
                 "gate_up": Linear(ops.interleave_gate_up(g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight"))),
                 "down": Linear(g(p + "mlp.down_proj.weight"))}
            if kind == "linear_attention":
                a = p + "linear_attn."
                w = torch.cat([g(a + "in_proj_qkv.weight"), g(a + "in_proj_z.weight"), g(a + "in_proj_b.weight"),
                               g(a + "in_proj_a.weight")])
                pad = (-w.shape[0]) % 64  # keep the output row stride 16-byte aligned
                if pad:
                    w = torch.cat([w, w.new_zeros(pad, w.shape[1])])
                L.update(in_proj=Linear(w), conv=g(a + "conv1d.weight").reshape(self.conv_dim, self.kconv).contiguous(),
                         dt_bias=g32(a + "dt_bias"), a_log=g32(a + "A_log"), gnorm=g(a + "norm.weight"),
                         out_proj=Linear(g(a + "out_proj.weight")))
                self.delta_index[i] = len(self.delta_index)
            else:
                a = p + "self_attn."
                L.update(qkv=Linear(torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")])),
                         o=Linear(g(a + "o_proj.weight")), q_norm=g(a + "q_norm.weight"),
                         k_norm=g(a + "k_norm.weight"))
                self.attn_index[i] = len(self.attn_index)
            self.layers.append(L)
        self.inv_freq = self.frequencies(c).to(self.device)
        self.pool = None

    @staticmethod
    def frequencies(c):
        rp = c.get("rope_parameters") or {"rope_theta": c.get("rope_theta", 10000.0)}
        dim = int(c["head_dim"] * rp.get("partial_rotary_factor", 1.0))
        return 1.0 / (rp["rope_theta"] ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))

    def kv_layout(self):
        return len(self.attn_index), self.hkv, self.d

    def recurrent_layout(self):
        return len(self.delta_index), self.kconv - 1, self.conv_dim, self.hv, self.dk, self.dv

    def _recurrent(self, segments, n):
        lay = getattr(segments, "recurrent", None)
        if lay is None or lay.n_rows != n:
            lay = RecurrentLayout.build(segments, n, self.kconv - 1, self.device)
            lay.choose_lead(self.hv)
            segments.recurrent = lay
        return lay

    # ------------------------------------------------------------------ forward
    def hidden(self, ids, positions, segments):
        """Final-normed (zero-centred) hidden states [N, hidden] bf16 (qwen3_5.py:410-417); the
        runner uses ``residual`` and norms only the read rows in the readout kernel."""
        return ops.rms_norm(self.residual(ids, positions, segments), self.norm, self.eps, zero_centered=True)

    def residual(self, ids, positions, segments, saves=None):
        """Residual-stream states [N, hidden] after the last layer (before the final norm)."""
        n = ids.shape[0]
        x = ops.embed(ids, self.embed_tokens)
        table = ops.rope_table(positions, self.inv_freq)
        lay = layout_of(segments, n, self.device)
        rl = self._recurrent(segments, n) if self.delta_index else None
        scratch = _lib.delta_scratch(rl.n_chunks, self.hk, self.hv, self.device) if rl is not None else None
        for i, L in enumerate(self.layers):
            hn = ops.rms_norm(x, L["in_norm"], self.eps, zero_centered=True)
            if L["kind"] == "linear_attention":
                self._deltanet(i, L, hn, x, rl, scratch)
            else:
                self._attention(i, L, hn, x, table, lay, saves)
            hn = ops.rms_norm(x, L["post_norm"], self.eps, zero_centered=True)
            act = ops.linear_swiglu(hn, L["gate_up"].w)
            ops.linear(act, L["down"].w, residual=x)
        return x

    def _deltanet(self, i, L, hn, x, rl, scratch):
        n = hn.shape[0]
        li = self.delta_index[i]
        kd, vd, hv, C = self.hk * self.dk, self.hv * self.dv, self.hv, self.conv_dim
        P = ops.linear(hn, L["in_proj"].w)
        qkv, z = P[:, :C], P[:, C:C + vd]
        b, a = P[:, C + vd:C + vd + hv], P[:, C + vd + hv:C + vd + 2 * hv]
        pool = self.pool
        hist = pool.conv[li].view(-1, C) if (pool is not None and pool.n_slots) else None
        conv = torch.empty(n, C, dtype=torch.bfloat16, device=self.device)
        _lib.call("dan_causal_conv", _lib.ptr(qkv), P.stride(0), _lib.ptr(hist), C if hist is not None else 0,
                  _lib.ptr(L["conv"]), _lib.ptr(rl.prev), _lib.ptr(conv), C, n, C, _lib.stream())
        if rl.tail_dst and hist is not None:  # conv tails at the save cuts -> pool slots
            k1 = self.kconv - 1
            tails = torch.empty(len(rl.tail_dst) * k1, C, dtype=torch.bfloat16, device=self.device)
            _lib.call("dan_gather_rows", _lib.ptr(qkv), P.stride(0), _lib.ptr(hist), C, _lib.ptr(rl.tail_codes),
                      tails.shape[0], _lib.ptr(tails), C, C, _lib.stream())
            for j, slot in enumerate(rl.tail_dst):
                pool.conv[li, slot].copy_(tails[j * k1:(j + 1) * k1])
        state = pool.state[li] if (pool is not None and pool.n_slots) else None
        out = torch.empty(n, vd, dtype=torch.bfloat16, device=self.device)
        _lib.call("dan_gated_delta_scan", _lib.ptr(conv[:, :kd]), _lib.ptr(conv[:, kd:2 * kd]), _lib.ptr(conv[:, 2 * kd:]),
                  C, _lib.ptr(b), _lib.ptr(a), P.stride(0), _lib.ptr(L["a_log"]), _lib.ptr(L["dt_bias"]),
                  _lib.ptr(rl.segs), rl.n_segs, _lib.ptr(rl.branches), _lib.ptr(rl.chunks), rl.n_chunks,
                  _lib.ptr(state), state.stride(0) if state is not None else 0, _lib.ptr(out), vd, self.hk, hv,
                  self.dk, self.dv, float(self.dk ** -0.5), _lib.ptr(scratch), scratch.numel(), *rl.lead,
                  _lib.ptr(_lib.status_word(self.device)), _lib.stream(),
                  work=n * (2 * kd + vd) * 2 + n * hv * 2 * 2 + n * vd * 2 + rl.n_state_io * hv * self.dk * self.dv * 4)
        y = torch.empty_like(out)
        _lib.call("dan_gated_rms_norm", _lib.ptr(out), vd, _lib.ptr(z), P.stride(0), _lib.ptr(L["gnorm"]),
                  float(self.eps), _lib.ptr(y), vd, n, hv, self.dv, _lib.stream())
        ops.linear(y, L["out_proj"].w, residual=x)

    def _attention(self, i, L, hn, x, table, lay, saves):
        n = hn.shape[0]
        h, hkv, d = self.h, self.hkv, self.d
        qkv = ops.linear(hn, L["qkv"].w)
        qg = qkv[:, :h * 2 * d].view(n, h, 2 * d)
        q, gate = qg[:, :, :d], qg[:, :, d:]
        k = qkv[:, h * 2 * d:h * 2 * d + hkv * d].view(n, hkv, d)
        v = qkv[:, h * 2 * d + hkv * d:].view(n, hkv, d)
        ops.rms_norm(q, L["q_norm"], self.eps, zero_centered=True, out=q)
        ops.rms_norm(k, L["k_norm"], self.eps, zero_centered=True, out=k)
        ops.rope_(q, table, self.rot)
        ops.rope_(k, table, self.rot)
        ai = self.attn_index[i]
        if saves is not None and self.pool is not None:
            ops.kv_store(k, v, self.pool.k[ai], self.pool.v[ai], saves[0], saves[1])
        ao = torch.empty(n, h * d, dtype=torch.bfloat16, device=self.device)
        tree_attention(q, k, v, lay, out=ao.view(n, h, d), pool=self.pool, layer=ai)
        ops.sigmoid_gate_(ao, gate, d)
        ops.linear(ao, L["o"].w, residual=x)

    def readout(self, x, read_rows, label_ids, offsets, max_labels):
        return ops.label_readout(x, read_rows, self.norm, self.eps, ops.NORM_ZERO_CENTERED, self.lm_head, label_ids,
                                 offsets, max_labels)

    def label_logits(self, h, label_ids):
        """fp32 logits of ``label_ids`` for one final-normed hidden state (qwen3_5.py:419-420)."""
        return _label_logits(self, h, label_ids)

    def linear_params(self):
        c, hd = self.config, self.config["hidden_size"]
        total = 0
        for L in self.layers:
            total += 3 * hd * c["intermediate_size"]
            if L["kind"] == "linear_attention":
                total += hd * (self.conv_dim + self.hv * self.dv + 2 * self.hv) + self.hv * self.dv * hd
            else:
                total += hd * (self.h * 2 * self.d + 2 * self.hkv * self.d) + self.h * self.d * hd
        return total
