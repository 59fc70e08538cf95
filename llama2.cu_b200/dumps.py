"""Logit-dump and token-id files in the reference's formats.

The reference's generate loop, built with -DDUMP_LOGITS, appends every
sampled step's fp32 logits row to a raw binary file (llama2_cublas.cu:5886-5894:
fwrite of vocab_size floats per step, "wb" for the first step and "ab" after)
and the sampled ids to a JSON list (llama2_cublas.cu:5908-5913); its analysis
script reads the logits back as raw float32 reshaped to (steps, vocab) or
from .npy (precision_ablation.py:319-333) and the ids with json.load
(precision_ablation.py:568-570).  These helpers write and read the same
files from the batched sampler's outputs (device tensors are copied to the
host), so the reference's KL / MSE / perplexity tooling reads them unchanged.
"""
import json
import os

import numpy as np


def _host_rows(logits):
    if hasattr(logits, "detach"):  # torch tensor (CPU or CUDA)
        logits = logits.detach().float().cpu().numpy()
    a = np.ascontiguousarray(logits, dtype=np.float32)
    return a.reshape(1, -1) if a.ndim == 1 else a


def append_logits(path, logits, first=False):
    """Appends rows [steps, vocab] (or one row) of fp32 logits to a raw
    binary dump; `first` truncates the file first (the reference's step 0)."""
    rows = _host_rows(logits)
    with open(path, "wb" if first else "ab") as f:
        f.write(rows.tobytes())
    return rows.shape[0]


def save_logits_npy(path, logits):
    """The .npy form the analysis script prefers: shape (steps, vocab)."""
    np.save(path, _host_rows(logits))


def load_logits(path, vocab):
    """Rows of a dump: .npy as stored, raw binary as (steps, vocab) with a
    trailing partial row dropped."""
    if str(path).endswith(".npy"):
        return np.load(path)
    raw = np.fromfile(path, dtype=np.float32)
    n = raw.size // vocab
    return raw[: n * vocab].reshape(n, vocab)


def append_token_ids(path, ids, first=False):
    """Appends sampled ids to the JSON id list (rewritten as a complete list,
    so json.load always reads it)."""
    if hasattr(ids, "detach"):
        ids = ids.detach().cpu().numpy()
    ids = [int(i) for i in np.asarray(ids).reshape(-1)]
    old = [] if first or not os.path.exists(path) else load_token_ids(path)
    with open(path, "w") as f:
        f.write("[" + ",".join(str(i) for i in old + ids) + "]")
    return len(old) + len(ids)


def load_token_ids(path):
    with open(path) as f:
        text = f.read().strip()
    if text and not text.endswith("]"):  # the reference's writer leaves the list open
        text += "]"
    return json.loads(text) if text else []
