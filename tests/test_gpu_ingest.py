"""Weight ingestion and the on-disk MX format, through libmxq.so's C-ABI:

- MXQW files (mxq_weight_save / mxq_weight_load) round-trip the MX bytes
  exactly, and a loaded weight computes the same linear bit for bit;
- a GGUF file (the `gguf` package the reference's training/gguf_translator.py
  reads with; Q8_0 and F32 tensors written here, none ships with the
  reference) and a torch state dict are ingested as exactly mx_quantize_w of
  their fp32 values (checked against the oracle's quantiser).
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from cpu_model_b200 import ingest, mx, synth

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("fmt,n,k", [(4, 300, 4096), (8, 77, 96)])
def test_mxqw_roundtrip(ctx, tmp_path, fmt, n, k):
    w, ws = synth.weights(fmt, n, k, -9, -2, 7 + n)
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)
    path = tmp_path / "w.mxqw"
    W.save(path)
    raw = path.read_bytes()
    assert raw[:4] == b"MXQW" and len(raw) == 32 + w.nbytes + ws.nbytes
    W2 = mx.MXWeight.load(path, ctx)
    assert (W2.fmt, W2.n, W2.k) == (fmt, n, k)
    d2, s2 = W2.download()
    assert np.array_equal(d2, w) and np.array_equal(s2, ws)
    x = cuda(synth.normal((3, k), 8))
    assert np.array_equal(host(mx.mx_linear(x, W, ctx)), host(mx.mx_linear(x, W2, ctx)))
    W.close()
    W2.close()


def test_mxqw_rejects_bad_files(ctx, tmp_path):
    bad = tmp_path / "bad.mxqw"
    bad.write_bytes(b"NOPE" + bytes(60))
    with pytest.raises(ValueError):
        mx.MXWeight.load(bad, ctx)
    w, ws = synth.weights(8, 8, 64, -8, -3, 1)
    W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 8, 8, 64, ctx)
    W.save(tmp_path / "t.mxqw")
    trunc = (tmp_path / "t.mxqw").read_bytes()[:-5]
    (tmp_path / "trunc.mxqw").write_bytes(trunc)
    with pytest.raises(ValueError):
        mx.MXWeight.load(tmp_path / "trunc.mxqw", ctx)
    W.close()


@pytest.mark.parametrize("fmt", [4, 8])
def test_gguf_ingest(ctx, tmp_path, fmt):
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(3)
    a = rng.standard_normal((96, 512)).astype(np.float32)
    b = (rng.standard_normal((40, 100)) * 0.1).astype(np.float32)          # rows not a multiple of 32
    path = str(tmp_path / "m.gguf")
    wr = gguf.GGUFWriter(path, arch="llama")
    wr.add_tensor("blk.0.ffn_up.weight", gguf.quants.quantize(a, gguf.GGMLQuantizationType.Q8_0),
                  raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    wr.add_tensor("blk.0.small", b)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    assert set(ingest.gguf_tensor_names(path)) == {"blk.0.ffn_up.weight", "blk.0.small"}
    reader = gguf.GGUFReader(path)
    for t in reader.tensors:
        vals = np.asarray(gguf.quants.dequantize(t.data, t.tensor_type), np.float32).reshape(-1, int(t.shape[0]))
        kp = (vals.shape[1] + 31) // 32 * 32
        vals = np.pad(vals, ((0, 0), (0, kp - vals.shape[1])))
        W = ingest.from_gguf(path, t.name, fmt, ctx)
        d, s = W.download()
        d0, s0, _ = oracle.quantize_w(fmt, vals)
        assert np.array_equal(d, d0) and np.array_equal(s, s0)
        W.close()


def test_torch_state_ingest(ctx, tmp_path):
    g = torch.Generator().manual_seed(5)
    state = {"proj.weight": torch.randn(64, 1616, generator=g) * 0.05, "bias": torch.zeros(64)}
    torch.save(state, tmp_path / "s.pt")
    W = ingest.from_torch(str(tmp_path / "s.pt"), "proj.weight", mx.FMT_INT8, ctx)
    vals = np.pad(state["proj.weight"].numpy(), ((0, 0), (0, 1632 - 1616)))
    d0, s0, _ = oracle.quantize_w(8, vals)
    d, s = W.download()
    assert np.array_equal(d, d0) and np.array_equal(s, s0)
    with pytest.raises(ValueError):
        ingest.from_torch(state, "bias", mx.FMT_INT8, ctx)
    W.close()
