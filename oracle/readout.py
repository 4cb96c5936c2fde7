"""The option-code readout on the CPU in numpy -- test infrastructure only (see oracle/__init__.py).

Restates basal/readout.py (rkinas/basal 2.8.1):
  capped(z, softcap)          readout.py:39-41: softcap * tanh(z / softcap), or z
  rows(head_w, head_b, lids)  CodeReadout.rows, readout.py:57-69: fp32 rows of the sorted union of the prompts'
                              code ids, each prompt's columns into them, the padding mask
  logits(h, rows, softcap)    CodeReadout.logits, readout.py:71-74: fp32 h @ rows^T (+ bias), capped
  probs_of(z, idx, pad)       readout.py:76-79: gather, -inf at the padding, softmax per prompt
  probs(...) / probs_each(...) readout.py:81-104
The matmul order of numpy's BLAS differs from torch's; parity with the reference is to fp32 rounding.
"""
import numpy as np


def capped(z, softcap):
    z = np.asarray(z, np.float32)
    if not softcap:
        return z
    c = np.float32(softcap)
    return (np.tanh(z / c) * c).astype(np.float32)


def rows(head_w, head_b, lids):
    key = sorted({i for ids in lids for i in ids})
    W = np.asarray(head_w, np.float32)[key]
    b = None if head_b is None else np.asarray(head_b, np.float32)[key]
    col = {t: j for j, t in enumerate(key)}
    K = max(map(len, lids))
    idx = np.asarray([[col[i] for i in ids] + [0] * (K - len(ids)) for ids in lids], np.int64)
    pad = np.asarray([[False] * len(ids) + [True] * (K - len(ids)) for ids in lids])
    return (W, b), idx, pad


def logits(h, rws, softcap=None):
    W, b = rws
    z = np.asarray(h, np.float32) @ W.T
    return capped(z if b is None else z + b, softcap)


def softmax(z):
    z = np.asarray(z, np.float32)
    m = z.max(-1, keepdims=True)
    e = np.exp(z - m)
    return (e / e.sum(-1, keepdims=True)).astype(np.float32)


def probs_of(z, idx, pad):
    g = np.take_along_axis(np.asarray(z, np.float32), idx, 1)
    g = np.where(pad, np.float32(-np.inf), g)
    return softmax(g)


def probs(head_w, head_b, h, lids, softcap=None):
    rws, idx, pad = rows(head_w, head_b, lids)
    p = probs_of(logits(h, rws, softcap), idx, pad)
    return [row[: len(ids)].tolist() for row, ids in zip(p, lids)]


def probs_each(head_w, head_b, h, lids, softcap=None):
    out = []
    for r, ids in enumerate(lids):
        W = np.asarray(head_w, np.float32)[list(ids)]
        b = None if head_b is None else np.asarray(head_b, np.float32)[list(ids)]
        out.append(softmax(logits(np.asarray(h, np.float32)[r][None], (W, b), softcap))[0].tolist())
    return out
