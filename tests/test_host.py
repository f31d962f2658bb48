"""CPU tests of the host side: GGUF I/O, quantisers, config, the C ABI
library's symbols, factories and error behaviour (no GPU needed)."""

from __future__ import annotations

import hashlib
import re

import numpy as np
import pytest
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.gguf import GGML_F32, GGML_Q8_0, GGUFFile, GGUFWriter
from breezetoken_b200.model import Qwen35Config
from breezetoken_b200.quant import dequantize_q8_0, iq3s_grid, quantize_iq3_s, quantize_q8_0
from breezetoken_b200.synth import QWEN35_TINY, qwen35_tensors, write_qwen35_gguf
from oracle.dequant import dequant_iq3_s
from tests.conftest import ROOT

IQ3S_SHA256 = "bd1af4945a1717c65610b0284e4628b9a1ba3b306fae3a06f6e5f597356e349f"


def test_library_exports_every_declared_symbol() -> None:
    header = (ROOT / "include" / "bt_b200.h").read_text()
    declared = set(re.findall(r"BT_API\s+[\w\s\*]+?\b(bt_\w+)\s*\(", header))
    assert declared == set(N.EXPORTED)
    lib = N.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.bt_version() >= 100
    assert lib.bt_q8_row_bytes(1024) == 1088
    assert lib.bt_q8_row_bytes(3584) == 3808
    assert lib.bt_q8_row_bytes(32) == 16 + 32


def test_c_abi_rejects_bad_arguments_without_a_gpu() -> None:
    lib = N.load()
    assert lib.bt_linear_q8(None, None, None, 4, 32, 1, None) == N.BT_ERR_INVALID
    assert b"null" in lib.bt_last_error()
    assert lib.bt_linear_q8(1, 1, 1, 4, 32, 3, None) == N.BT_ERR_UNSUPPORTED
    assert lib.bt_gdn_decode(1, 1, 1, N.BT_F32, 1, 1, 1, 1, 1, 3, 16, 128, 1.0, 1e-6, None) == N.BT_ERR_INVALID
    assert lib.bt_attention_workspace_bytes(1, 2, 8, 256, 4) > 0
    with pytest.raises(N.B200Error):
        N.call("bt_repack_q8_0", None, None, 1, 32, 0, 1, None)


def test_iq3s_codebook_pinned() -> None:
    grid = iq3s_grid()
    assert grid.shape == (512, 4)
    assert hashlib.sha256(grid.tobytes()).hexdigest() == IQ3S_SHA256
    assert np.array_equal(grid, np.load(ROOT / "oracle" / "iq3s_grid.npy"))
    assert set(np.unique(grid).tolist()) == {1, 3, 5, 7, 9, 11, 13, 15}


def test_gguf_roundtrip(tmp_path) -> None:
    w = GGUFWriter()
    w.add("general.architecture", "qwen35")
    w.add("x.int", 7)
    w.add("x.float", 1.5)
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    q = quantize_q8_0(np.linspace(-1, 1, 64, dtype=np.float32).reshape(2, 32))
    w.add_tensor("a", (3, 4), GGML_F32, a)
    w.add_tensor("q", (2, 32), GGML_Q8_0, q)
    path = w.write(tmp_path / "t.gguf")
    with GGUFFile(path) as g:
        assert g.arch == "qwen35" and g.metadata["x.int"] == 7 and g.metadata["x.float"] == 1.5
        assert g.tensor_info("a") == ((3, 4), "f32")
        assert np.array_equal(g.f32("a"), a)
        assert np.array_equal(g.raw("q"), q.reshape(-1))
        with pytest.raises(KeyError):
            g.tensor_layout("missing")
        with pytest.raises(NotImplementedError):
            g.f32("q")
    g = GGUFFile(path)
    g.close()
    with pytest.raises(ValueError, match="closed"):
        g.raw("a")


def test_gguf_rejects_corrupt_files(tmp_path) -> None:
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + bytes(60))
    with pytest.raises(ValueError):
        GGUFFile(bad)
    v2 = tmp_path / "v2.gguf"
    v2.write_bytes(b"GGUF" + (2).to_bytes(4, "little") + bytes(16))
    with pytest.raises(ValueError, match="version"):
        GGUFFile(v2)
    good = write_qwen35_gguf(tmp_path / "tiny.gguf", QWEN35_TINY, seed=1)
    data = good.read_bytes()
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(data[: len(data) // 2])
    with pytest.raises(ValueError):
        GGUFFile(trunc)


def test_reference_reader_parses_our_files(tiny_gguf) -> None:
    """The writer's output is what the reference reader expects: names, shapes, types."""
    with GGUFFile(tiny_gguf) as g:
        names = g.tensor_names()
        assert names == [n for n, _, _ in qwen35_tensors(QWEN35_TINY)]
        assert g.tensor_info("token_embd.weight") == ((QWEN35_TINY.vocab, QWEN35_TINY.hidden), "q8_0")
        assert g.tensor_info("blk.0.ssm_conv1d.weight") == ((3 * 2048, 4), "f32")
        assert (g.f32("blk.0.ssm_a") < 0).all()
        cfg = Qwen35Config.from_gguf(g, 512)
    assert cfg.attn_layers == (3,)
    assert cfg.max_context == 512 and cfg.rope_dim == 64 and cfg.vocab == 8192


def test_synth_deterministic(tmp_path) -> None:
    a = write_qwen35_gguf(tmp_path / "a.gguf", QWEN35_TINY, seed=5).read_bytes()
    b = write_qwen35_gguf(tmp_path / "b.gguf", QWEN35_TINY, seed=5).read_bytes()
    c = write_qwen35_gguf(tmp_path / "c.gguf", QWEN35_TINY, seed=6).read_bytes()
    assert a == b and a != c


def test_quantisers() -> None:
    rng = np.random.default_rng(0)
    x = rng.standard_normal((16, 512)).astype(np.float32) * 0.02
    q8 = dequantize_q8_0(quantize_q8_0(x), (16, 512))
    assert np.abs(q8 - x).max() <= np.abs(x).max() / 127 * 0.51 + 1e-7
    iq = dequant_iq3_s(quantize_iq3_s(x).reshape(-1), 16, 512)
    rel = np.linalg.norm(iq - x) / np.linalg.norm(x)
    assert rel < 0.35, rel  # 3.4 bits per weight
    assert np.array_equal(quantize_iq3_s(x), quantize_iq3_s(x))


def test_config_validation(tiny_gguf) -> None:
    with GGUFFile(tiny_gguf) as g:
        with pytest.raises(ValueError):
            Qwen35Config.from_gguf(g, 0)
        cfg = Qwen35Config.from_gguf(g, None)
    assert cfg.max_context == 8192


def test_make_backend_errors() -> None:
    from breezetoken_b200.backends import make_backend, resolve_device

    with pytest.raises(ValueError):
        make_backend("tilelang", "cuda")
    with pytest.raises(ValueError):
        resolve_device("cpu")
    with pytest.raises(ValueError):
        resolve_device("not-a-device")
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError):
            make_backend("b200", "cuda")


def test_uploader_cpu_copy_and_precision_measure(tmp_path) -> None:
    """The checkpoint uploader on a CPU device returns a copy of the bytes (a
    read-only memory map included); the precision report measures a planted
    error against the output scale and per element."""
    from breezetoken_b200.kernel_bench import _errors
    from breezetoken_b200.upload import Uploader

    rng = np.random.default_rng(62)
    blob = rng.integers(0, 256, 100_003, dtype=np.uint8)
    blob.tofile(tmp_path / "b.bin")
    mm = np.memmap(tmp_path / "b.bin", dtype=np.uint8, mode="r")
    up = Uploader("cpu")
    got = up.to_device(mm[3:])
    up.close()
    assert got.dtype == torch.uint8 and torch.equal(got, torch.from_numpy(blob[3:]))
    y = np.array([4.0, -2.0, 1.0, 1e-6], dtype=np.float32)
    want = y.astype(np.float64) - np.array([4e-6, 0.0, -1e-6, 5e-7])  # planted errors
    e = _errors(y, want, want.astype(np.float32))
    assert abs(e["rel_of_scale"] - 1e-6) < 1e-8  # 4e-6 of a scale of 4
    assert abs(e["rel_elem_max"] - 1e-6) < 1e-8  # the 1e-6 element is below 1e-3 of the scale
    assert e["host_f32_rel_of_scale"] < 1e-7 and e["elements"] == 4
