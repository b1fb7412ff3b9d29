"""Weight ingestion into MX weights: the two sources the reference's
training code reads, a GGUF file (training/gguf_translator.py:21,60, through
the `gguf` package) and a LibTorch / PyTorch tensor archive
(training/offline_trainer.cpp:105-128), plus the library's own MXQW file
(mxq_weight_save / mxq_weight_load).

Each tensor is brought to fp32 rows on the host by its source's own reader
(GGUF K-quants and Q8_0 are dequantised by `gguf`), moved to the device and
MX-quantised there (mx_quantize_w: E8M0 block scale per 32 elements, int8
or int4), so the ingested weight is exactly mx_quantize_w of the source's
fp32 values.  A tensor whose row length is not a multiple of 32 is
zero-padded on the right to the next multiple (the padding quantises to 0).
"""
import numpy as np
import torch

from . import mx


def _to_weight(rows, fmt, ctx):
    rows = np.ascontiguousarray(rows, np.float32)
    if rows.ndim == 1:
        rows = rows[None, :]
    rows = rows.reshape(rows.shape[0], -1)
    k = rows.shape[1]
    kp = (k + 31) // 32 * 32
    if kp != k:
        rows = np.pad(rows, ((0, 0), (0, kp - k)))
    return mx.MXWeight.from_float(torch.from_numpy(rows).cuda(), fmt, ctx)


def gguf_tensor_names(path):
    import gguf
    return [t.name for t in gguf.GGUFReader(path).tensors]


def from_gguf(path, name, fmt=mx.FMT_INT4, ctx=None):
    """One tensor of a GGUF file -> MXWeight [rows][cols] (GGUF stores the
    fastest-varying dimension first; rows = the remaining dimensions)."""
    import gguf
    reader = gguf.GGUFReader(path)
    for t in reader.tensors:
        if t.name == name:
            vals = gguf.quants.dequantize(t.data, t.tensor_type)
            cols = int(t.shape[0])
            return _to_weight(np.asarray(vals, np.float32).reshape(-1, cols), fmt, ctx)
    raise KeyError("tensor %r not in %s" % (name, path))


def from_torch(path_or_state, name, fmt=mx.FMT_INT4, ctx=None):
    """One 2-D tensor of a torch archive (torch.load of a state dict, or the
    dict itself) -> MXWeight."""
    state = path_or_state if isinstance(path_or_state, dict) else torch.load(path_or_state, map_location="cpu")
    t = state[name]
    if t.dim() != 2:
        raise ValueError("%s has %d dimensions; a linear weight has 2" % (name, t.dim()))
    return _to_weight(t.detach().float().cpu().numpy(), fmt, ctx)
