"""The GGUF reader (kq_gguf_* in include/kq.h, kernite_b200.gguf) against the GGML project's own
Python package gguf-py (0.19.0): files written by its GGUFWriter must read back with the same
tensor names, types, shapes, offsets and bytes that its GGUFReader reports; malformed files must
fail with KQ_E_INVALID and a reason, never crash. On the GPU, k-quant tensors loaded from a file
multiply through kq_matvec to the oracle's results and to gguf-py's own dequantisation.

The weights are the oracle's seeded synthetic blocks; gguf-py only writes and reads the file.
"""
import numpy as np
import pytest

import oracle

import kernite_b200 as kb
from kernite_b200.gguf import GGUFFile

gguf = pytest.importorskip("gguf")
T = gguf.GGMLQuantizationType

KQ_E_INVALID = 1001


def quant_bytes(qtype: int, rows: int, K: int, seed: int) -> np.ndarray:
    nb = K // 256
    blocks = oracle.fill(qtype, oracle.stream_key(seed, qtype), 0, rows * nb)
    return blocks.reshape(rows, nb * kb.block_bytes(qtype))


def write_model(path, alignment=None):
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_uint32("llama.block_count", 2)
    w.add_int64("test.negative", -5)
    w.add_float32("llama.attention.layer_norm_rms_epsilon", 1e-5)
    w.add_string("general.name", "kq-synthetic")
    w.add_array("test.array", [1, 2, 3])
    w.add_bool("test.flag", True)
    if alignment:
        w.add_custom_alignment(alignment)
    tensors = {
        "blk.0.attn_q.weight": (T.Q4_K, quant_bytes(4, 48, 512, 11)),
        "blk.0.ffn_down.weight": (T.Q6_K, quant_bytes(6, 40, 768, 12)),
        "blk.0.ffn_up.weight": (T.Q5_K, quant_bytes(5, 32, 512, 13)),
        "blk.1.attn_k.weight": (T.Q8_0, quant_bytes(8, 16, 512, 14)),
        "blk.1.attn_v.weight": (T.Q2_K, quant_bytes(2, 16, 256, 15)),
        "blk.1.ffn_gate.weight": (T.Q3_K, quant_bytes(3, 24, 512, 16)),
        "token_embd.weight": (None, np.arange(15, dtype=np.float32).reshape(3, 5)),
        "output_norm.weight": (None, np.linspace(-1, 1, 7).astype(np.float16)),
    }
    for name, (dtype, arr) in tensors.items():
        if dtype is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=dtype)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


@pytest.mark.parametrize("alignment", [None, 64])
def test_reader_agrees_with_gguf_py(tmp_path, alignment):
    path = tmp_path / "m.gguf"
    written = write_model(path, alignment)
    ref = {t.name: t for t in gguf.GGUFReader(str(path)).tensors}
    with GGUFFile(path) as f:
        got = {t.name: t for t in f.tensors()}
        assert list(got) == list(ref) == list(written)
        for name, t in got.items():
            r = ref[name]
            assert t.type == int(r.tensor_type), name
            assert t.shape == tuple(int(d) for d in r.shape), name
            assert t.offset == int(r.data_offset), name
            assert t.data.nbytes == int(r.n_bytes), name
            assert np.array_equal(t.data, np.asarray(r.data).reshape(-1).view(np.uint8)), name
            dtype, arr = written[name]
            assert np.array_equal(t.data, np.ascontiguousarray(arr).reshape(-1).view(np.uint8)), name
        q = f.tensor("blk.0.attn_q.weight")
        assert (q.qtype, q.rows, q.k) == (4, 48, 512)
        d = f.tensor("blk.0.ffn_down.weight")
        assert (d.qtype, d.rows, d.k) == (6, 40, 768)
        u = f.tensor("blk.0.ffn_up.weight")
        assert (u.qtype, u.rows, u.k) == (5, 32, 512)
        for name, ggml_type, rows, k in (("blk.1.attn_k.weight", 8, 16, 512),
                                         ("blk.1.attn_v.weight", 10, 16, 256),
                                         ("blk.1.ffn_gate.weight", 11, 24, 512)):
            t = f.tensor(name)
            assert (t.type, t.rows, t.k) == (ggml_type, rows, k), name
            with pytest.raises(kb.Error):  # decoded, not multiplied
                t.qtype
        assert f.meta_int("llama.block_count") == 2
        assert f.meta_int("test.negative") == -5
        assert f.meta_int("test.flag") == 1
        assert f.meta_str("general.name") == "kq-synthetic"
        assert f.meta_str("general.architecture") == "llama"
        if alignment:
            assert f.meta_int("general.alignment") == alignment
        with pytest.raises(kb.Error):
            f.tensor("no.such.tensor")
        with pytest.raises(kb.Error):
            f.meta_int("general.name")  # a string
        with pytest.raises(kb.Error):
            f.tensor("token_embd.weight").qtype


def test_malformed_files_are_rejected(tmp_path):
    good = tmp_path / "m.gguf"
    write_model(good)
    blob = good.read_bytes()
    bad = tmp_path / "bad.gguf"
    cases = {
        "magic": b"GGUX" + blob[4:],
        "version": blob[:4] + (7).to_bytes(4, "little") + blob[8:],
        "huge count": blob[:8] + (2**62).to_bytes(8, "little") + blob[16:],
    }
    # every truncation point inside the header and tensor table, and inside the data (the file
    # may end in padding after the last tensor, which is not data)
    data_end = max(int(t.data_offset) + int(t.n_bytes) for t in gguf.GGUFReader(str(good)).tensors)
    for cut in list(range(0, 600, 7)) + [data_end - 1, data_end - 500]:
        cases[f"cut {cut}"] = blob[:cut]
    for what, data in cases.items():
        bad.write_bytes(data)
        with pytest.raises(kb.Error) as e:
            GGUFFile(bad)
        assert e.value.code in (KQ_E_INVALID, 1002), what
        assert e.value.message, what
    with pytest.raises(kb.Error):
        GGUFFile(tmp_path / "missing.gguf")


@pytest.mark.gpu
def test_gguf_weights_multiply_like_the_oracle_and_gguf_py(tmp_path):
    import torch

    path = tmp_path / "m.gguf"
    write_model(path)
    kernels = kb.Kernels.load(0)
    with GGUFFile(path) as f:
        for name in ("blk.0.attn_q.weight", "blk.0.ffn_down.weight", "blk.0.ffn_up.weight"):
            t = f.tensor(name)
            W = t.to_device()
            x = np.random.default_rng(5).standard_normal((1, t.k), dtype=np.float32)
            y = torch.zeros((1, t.rows), dtype=torch.float32, device="cuda")
            kernels.matvec(t.qtype, y, W, torch.from_numpy(x).cuda(), t.rows, t.k, 1)
            torch.cuda.synchronize()
            y = y.cpu().numpy()
            y_ref, bound = oracle.matvec_ref(t.qtype, np.array(t.data), x, t.k, 0, t.rows)
            assert (np.abs(y - y_ref) <= 1e-3 * bound).all(), name
            # gguf-py's own decode of the same bytes, in f64
            wf = gguf.quants.dequantize(np.array(t.data).reshape(t.rows, -1), T(t.type))
            y_gg = wf.astype(np.float64) @ x[0].astype(np.float64)
            assert (np.abs(y[0] - y_gg) <= 1e-3 * bound[0]).all(), name


@pytest.mark.gpu
def test_gguf_weights_decode_like_gguf_py(tmp_path):
    import torch

    path = tmp_path / "m.gguf"
    write_model(path)
    kernels = kb.Kernels.load(0)
    with GGUFFile(path) as f:
        for name in ("blk.0.attn_q.weight", "blk.0.ffn_down.weight", "blk.0.ffn_up.weight",
                     "blk.1.attn_k.weight", "blk.1.attn_v.weight", "blk.1.ffn_gate.weight"):
            t = f.tensor(name)
            n = t.rows * t.k // 256
            out = torch.empty(n * 256, dtype=torch.float32, device="cuda")
            kernels.dequant(t.type, out, t.to_device(), n)
            torch.cuda.synchronize()
            want = gguf.quants.dequantize(np.array(t.data).reshape(t.rows, -1), T(t.type))
            want = np.ascontiguousarray(want, dtype=np.float32).reshape(-1)
            assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32)), name
