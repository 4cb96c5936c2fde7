"""The readout of the option codes, B200 build (the interface of basal/readout.py, rkinas/basal 2.8.1).

A question's answer is the softmax over its option codes of the logits at the answer position; only those rows of
the output head are read. Here they are read straight from the head (bf16) by id inside the contraction kernel
(basal::code_logits): nothing is copied or widened to fp32 first, so the row cache keeps only the ids. Products and sums are fp32; every logit is one fixed-order sum, so a prompt's probabilities are the same bits
whatever prompts are read with it (probs and probs_each agree exactly).

  rows(lids) -> (rows, idx, pad)   rows = (ids of the union of the prompts' codes on the device, None): the bias, if
                                   any, is read by id from the head inside the kernel as well
  logits(h, rows) -> fp32 [n, k]   basal::code_logits, soft cap applied once
  probs_of(z, idx, pad)            basal::code_probs: gather, -inf padding, softmax
  device_probs(h, rows, idx, pad)  probs_of(logits(h, rows), idx, pad): the device part of probs
  probs(h, lids), probs_each(h, lids)   device_probs, then one copy to the host
"""
import torch

from . import ops

WROWS_BYTES = 64 << 20  # what an engine's code-row cache may hold (here: the ids, 8 bytes a code)


def _size(x):
    """Bytes held by a cache entry: a tensor, None, or a tuple of them."""
    if isinstance(x, tuple):
        return sum(map(_size, x))
    return 0 if x is None else int(x.nbytes)


def code_rows(cache, key, make):
    """cache[key], made by make() when missing. The cache (a dict: insertion order = use order, newest last) keeps
    the most recently used entries whose bytes fit within WROWS_BYTES; the entry just used always stays
    (basal/readout.py:23-36)."""
    entry = cache.pop(key) if key in cache else make()
    cache[key] = entry
    excess = sum(_size(v) for v in cache.values()) - WROWS_BYTES
    while excess > 0 and len(cache) > 1:
        excess -= _size(cache.pop(next(iter(cache))))
    return entry


def capped(z, softcap):
    """The model's final logit soft cap (Gemma: softcap x tanh(z / softcap)), applied once; none: z as it is."""
    if not softcap:
        return z
    return softcap * torch.tanh(z / softcap)


class CodeReadout:
    """The code readout of one output head (an nn.Linear-like module: weight [vocab, D], optional bias) and soft cap."""

    def __init__(self, head, softcap=None, cache=None, to_dev=None):
        self.head, self.softcap = head, softcap
        self.cache = {} if cache is None else cache
        self.to_dev = to_dev or (lambda x: x.to(head.weight.device))

    def rows(self, lids):
        """(rows, idx, pad) for prompts whose option ids are lids: rows = (the sorted union of the ids on the device,
        None); idx [n, widest] = each prompt's columns into that union, pad = True past a prompt's own count."""
        union = tuple(sorted(set().union(*lids)))
        rows = code_rows(self.cache, union, lambda: (self.to_dev(torch.tensor(union, dtype=torch.int64)), None))
        column = {code: j for j, code in enumerate(union)}
        width = max(len(ids) for ids in lids)
        idx = torch.zeros(len(lids), width, dtype=torch.int64)
        pad = torch.ones(len(lids), width, dtype=torch.bool)
        for r, ids in enumerate(lids):
            idx[r, :len(ids)] = torch.tensor([column[i] for i in ids], dtype=torch.int64)
            pad[r, :len(ids)] = False
        return rows, self.to_dev(idx), self.to_dev(pad)

    def logits(self, h, rows):
        ids, _ = rows
        b = getattr(self.head, "bias", None)
        return ops.code_logits(h, self.head.weight, ids, b, float(self.softcap or 0.0))

    @staticmethod
    def probs_of(z, idx, pad):
        """Code logits [n, k] -> each prompt's probabilities over its codes [n, K] (padding 0), as a tensor."""
        return ops.code_probs(z, idx, pad)

    def device_probs(self, h, rows, idx, pad):
        """probs_of(logits(h, rows), idx, pad): the probabilities [n, K] as a device tensor."""
        return self.probs_of(self.logits(h, rows), idx, pad)

    def probs(self, h, lids):
        rows, idx, pad = self.rows(lids)
        p = self.device_probs(h, rows, idx, pad).tolist()  # one device sync
        return [row[: len(ids)] for row, ids in zip(p, lids)]

    def probs_each(self, h, lids):
        """probs, each prompt as if read alone: the kernels' results do not depend on the other prompts, so this is
        probs itself (basal/readout.py:86-104 reads each prompt with its own product for that guarantee)."""
        return self.probs(h, lids)
