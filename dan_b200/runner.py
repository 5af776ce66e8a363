"""Packed, prefill-only reads on the dan_b200 kernels (dan/runner.py:1-94).

Any number of read plans run in one forward pass: each plan contributes its
prompt (trunk) followed by one branch per question; the tree-attention kernel
keeps questions apart. Branch positions continue from the end of their trunk.
A plan whose static prefix is in the prefix pool starts from its cached
pages and computes only the rest of its prompt.

``pack`` reproduces the reference's packing exactly (ids, positions,
segments, read rows, stores); ``forward`` uploads one batch, runs the model,
and reads every question's label logits and probabilities with one fused
readout kernel; ``read_many`` copies them to the host once per batch.
``submit`` / ``read_stream`` keep a batch queued on the device while the host
packs the next one.
"""
import numpy as np
import torch

from . import _lib
from .attention import Batch, segment
from .cache import PrefixPool
from .loader import load


def _upload(xs, dtype, device):
    t = torch.as_tensor(np.asarray(xs), dtype=dtype)
    return t.pin_memory().to(device, non_blocking=True)


class Runner:
    def __init__(self, model, device="cuda", dtype=torch.bfloat16, cache_bytes=2 << 30, adapter=None,
                 quantization=None, merge_projections=True):
        """``model``: a model directory or an already-built model. ``adapter`` (LoRA) must be
        merged into the checkpoint beforehand: serving runs merged weights (runner.py:23-26)."""
        if adapter:
            raise NotImplementedError("merge LoRA adapters into the checkpoint before serving on dan_b200")
        if not torch.cuda.is_available():
            raise RuntimeError("dan_b200 needs a CUDA GPU (sm_100a); it has no CPU path")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.model = load(model, self.device, dtype, quantization)
        self.cache = None
        if cache_bytes:
            rec = getattr(self.model, "recurrent_layout", lambda: None)()
            layers, hkv, d = self.model.kv_layout()
            self.cache = PrefixPool(cache_bytes, layers, hkv, d, self.device, rec)
        self.model.pool = self.cache

    def pack(self, plans, use_cache=True):
        """Flat ids and positions, one segment per plan with questions, the read rows
        with their label ids, and the static prefixes to store (runner.py:38-64)."""
        ids, pos, segs, reads, stores = [], [], Batch(), [], []
        use_cache = use_cache and self.cache is not None
        for plan in plans:
            if not plan.branches:
                continue
            static = plan.prefix[:plan.static]
            past = self.cache.get(static) if use_cache and static else None
            skip = plan.static if past else 0
            start = len(ids)
            trunk = plan.prefix[skip:]
            ids += trunk
            pos += range(skip, len(plan.prefix))
            branch = [0] * len(trunk)
            for j, b in enumerate(plan.branches, 1):
                ids += b.suffix
                pos += range(len(plan.prefix), len(plan.prefix) + len(b.suffix))
                branch += [j] * len(b.suffix)
                reads.append((len(ids) - 1, b.label_ids))
            save = plan.static if use_cache and static and not past else 0
            segs.append(segment(start, branch, past, save, skip, self.device))
            if save:
                stores.append((static, segs[-1]))
        return ids, pos, segs, reads, stores

    def _reserve(self, segs, stores):
        """Pool pages for this batch's prefix saves; returns [(static, seg, entry)] and the
        (src_rows, dst_rows) row lists of the K/V copies."""
        pinned = [s.past for s in segs if s.past]
        out, src, dst, taken = [], [], [], set()
        for static, seg in stores:
            key = tuple(static)
            entry = None if key in taken else self.cache.reserve(static, seg.save, pinned)
            taken.add(key)
            if entry is None:
                seg.save = 0
                continue
            pinned.append(entry)
            seg.save_entry = entry
            out.append((static, seg, entry))
            src += range(seg.start, seg.start + seg.save)
            dst += self.cache.rows(entry, seg.save)
        return out, src, dst

    def forward_flat(self, plans, use_cache=True):
        """(logits, probs, offsets): flat fp32 device tensors over every question's labels
        in plan order, and the host offsets of each question's slice."""
        ids, pos, segs, reads, stores = self.pack(plans, use_cache)
        offsets = np.zeros(len(reads) + 1, dtype=np.int64)
        if not reads:
            z = torch.empty(0, device=self.device)
            return z, z, offsets
        dev = self.device
        held, src, dst = self._reserve(segs, stores) if stores else ([], [], [])
        try:
            ids_t = _upload(ids, torch.int64, dev)
            pos_t = _upload(pos, torch.int64, dev)
            saves = (_upload(src, torch.int32, dev), _upload(dst, torch.int32, dev)) if src else None
            labels = [list(l) for _, l in reads]
            offsets[1:] = np.cumsum([len(l) for l in labels])
            read_rows = _upload([r for r, _ in reads], torch.int32, dev)
            label_ids = _upload([x for l in labels for x in l], torch.int32, dev)
            off_t = _upload(offsets.astype(np.int32), torch.int32, dev)
            model = self.model
            state = model.residual(ids_t, pos_t, segs, saves)
            logits, probs = model.readout(state, read_rows, label_ids, off_t, max(len(l) for l in labels))
        except Exception:
            for _, _, entry in held:
                self.cache.release(entry)
            raise
        for static, seg, entry in held:
            self.cache.commit(static, entry)
        return logits, probs, offsets

    def forward(self, plans, use_cache=True):
        """Per plan, per branch: the fp32 logits of its label tokens, on the device."""
        logits, _, offsets = self.forward_flat(plans, use_cache)
        flat = [logits[offsets[i]:offsets[i + 1]] for i in range(len(offsets) - 1)]
        return self._split(plans, flat)

    @torch.inference_mode()
    def submit(self, plans, probabilities=False):
        """Queue one batch: pack, upload, forward and the copy of its results into pinned
        host memory are all issued on the device's current stream without waiting for
        it; ``PendingRead.result()`` waits. Batches submitted back to back run in order,
        so the host packs the next batch while the device computes this one."""
        with torch.cuda.device(self.device):
            logits, probs, offsets = self.forward_flat(plans)
            stream = torch.cuda.current_stream(self.device)
            status = torch.empty(1, dtype=torch.int32, pin_memory=True)
            status.copy_(_lib.status_word(self.device), non_blocking=True)
            if logits.numel():
                host = torch.empty(2, logits.numel(), dtype=torch.float32, pin_memory=True)
                host.copy_(torch.stack([logits, probs]), non_blocking=True)
            else:
                host = torch.zeros(2, 0)
            done = torch.cuda.Event()
            done.record(stream)
        return PendingRead(self, plans, host, status, offsets, done, probabilities)

    def read_many(self, plans, probabilities=False):
        """Per plan, per branch: the logits of its label tokens (fp32, CPU), from one
        device-to-host copy per batch; with ``probabilities`` also the softmax of each.
        Runs on this runner's device whatever the calling thread's current device is."""
        return self.submit(plans, probabilities).result()

    def read_stream(self, batches, probabilities=False):
        """``read_many`` over an iterable of batches, yielding each batch's result in
        order while the next batch is already queued on the device (one in flight)."""
        pending = None
        for plans in batches:
            nxt = self.submit(plans, probabilities)
            if pending is not None:
                yield pending.result()
            pending = nxt
        if pending is not None:
            yield pending.result()

    @staticmethod
    def _split(plans, flat):
        out, k = [], 0
        for plan in plans:
            n = len(plan.branches)
            out.append(flat[k:k + n])
            k += n
        return out

    def read(self, plan):
        return self.read_many([plan])[0]


class PendingRead:
    """A submitted batch (``Runner.submit``): its results land in pinned host memory when
    the device reaches them. ``result()`` waits for that point only (not for batches
    queued after it), raises if a kernel of the device reported an error, and returns
    what ``read_many`` returns."""

    __slots__ = ("runner", "plans", "host", "status", "offsets", "done", "probabilities")

    def __init__(self, runner, plans, host, status, offsets, done, probabilities):
        self.runner, self.plans, self.host, self.status = runner, plans, host, status
        self.offsets, self.done, self.probabilities = offsets, done, probabilities

    def ready(self):
        return self.done.query()

    def result(self):
        self.done.synchronize()
        v = int(self.status[0])
        if v:
            with torch.cuda.device(self.runner.device):
                _lib.status_word(self.runner.device).zero_()
            raise RuntimeError(f"dan_b200 kernel error {v}: {_lib.STATUS_TEXT.get(v, 'unknown')}")
        both, off, plans = self.host, self.offsets, self.plans
        lg = [both[0, off[i]:off[i + 1]] for i in range(len(off) - 1)]
        out = Runner._split(plans, lg)
        if self.probabilities:
            pr = [both[1, off[i]:off[i + 1]] for i in range(len(off) - 1)]
            return out, Runner._split(plans, pr)
        return out
