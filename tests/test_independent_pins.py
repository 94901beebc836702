"""Pins of the block-quantised weights (GGUF Q8_0 / Q4_0) and of the GGUF file
reader that do not depend on this repository's own restatements.

The engine declares the Q8_0 / Q4_0 block formats (include/engine/dtype.hpp:95-125:
32 weights per block, one FP16 scale d; 34 and 18 bytes, tests/test_dtype.cpp:142-144)
and plans an mmap loader (include/engine/tensor.hpp:19-23), but ships neither a
kernel nor data for them.  The formats themselves are GGML's, published with
llama.cpp:

  Q8_0  { f16 d; int8 qs[32]; }       w[i] = d * qs[i]
  Q4_0  { f16 d; uint8 qs[16]; }      w[i] = d * ((qs[i] & 0xF) - 8),   i < 16
                                      w[i] = d * ((qs[i-16] >> 4) - 8), i >= 16

Three independent checks:
1. known-answer blocks assembled byte by byte below, with every expected weight
   written out from the definition above (nibble order, nibbles 0 and 15,
   negative, subnormal and maximal scales), against the C oracle (and, marked
   gpu, against the CUDA repack + GEMV through one-hot activations);
2. the `gguf` Python package (llama.cpp's gguf-py, version pinned below) as an
   independent quantiser / dequantiser, bit for bit against the oracle;
3. a GGUF file written by gguf-py's own GGUFWriter, read by the library's
   reader (csrc/gguf.cpp), and a file assembled field by field from the
   published layout in this test.
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

import oracle

gguf = pytest.importorskip("gguf")
GGUF_PY_VERSION = "0.19.0"  # the version these pins were written against

Q8_0, Q4_0 = 8, 4  # the oracle's / library's qtype codes
GGML_Q8_0, GGML_Q4_0 = 8, 2  # GGML type codes in a GGUF tensor table


def _h(bits: int) -> bytes:
    """An FP16 scale given by its bit pattern (little-endian)."""
    return struct.pack("<H", bits)


# FP16 bit patterns and their values, written out: 0x3800 = 2^-1, 0xBC00 = -1,
# 0x0001 = 2^-24 (smallest subnormal), 0x0003 = 3 * 2^-24, 0x7BFF = 65504 (largest
# finite), 0x4000 = 2, 0xB400 = -2^-2.
SCALES = {0x3800: 0.5, 0xBC00: -1.0, 0x0001: 2.0 ** -24, 0x0003: 3 * 2.0 ** -24,
          0x7BFF: 65504.0, 0x4000: 2.0, 0xB400: -0.25}


def q8_kat():
    """Four Q8_0 blocks (one row of K = 128) and their weights."""
    blocks, want = b"", []
    # block 0: d = 0.5, qs = 0, 1, -1, 127, -128, then 2..28
    qs = [0, 1, -1, 127, -128] + list(range(2, 29))
    blocks += _h(0x3800) + struct.pack("<32b", *qs)
    want += [0.5 * q for q in qs]
    # block 1: d = -1, every qs = 5
    blocks += _h(0xBC00) + struct.pack("<32b", *([5] * 32))
    want += [-5.0] * 32
    # block 2: d = 2^-24 (subnormal), qs[i] = i - 16
    qs = [i - 16 for i in range(32)]
    blocks += _h(0x0001) + struct.pack("<32b", *qs)
    want += [q * 2.0 ** -24 for q in qs]
    # block 3: d = 65504, qs alternate 1, -1, 0
    qs = [(1, -1, 0)[i % 3] for i in range(32)]
    blocks += _h(0x7BFF) + struct.pack("<32b", *qs)
    want += [65504.0 * q for q in qs]
    return np.frombuffer(blocks, np.uint8).copy(), np.array(want, np.float64)


def q4_kat():
    """Three Q4_0 blocks (one row of K = 96) and their weights."""
    blocks, want = b"", []
    # block 0: d = 2; byte j = j | (15 - j) << 4: element j has nibble j, element
    # j + 16 has nibble 15 - j (nibbles 0 and 15 both occur)
    qs = [j | ((15 - j) << 4) for j in range(16)]
    blocks += _h(0x4000) + bytes(qs)
    want += [2.0 * (j - 8) for j in range(16)] + [2.0 * ((15 - j) - 8) for j in range(16)]
    # block 1: d = -0.25, every byte 0x80: low nibbles 0 -> -8, high nibbles 8 -> 0
    blocks += _h(0xB400) + bytes([0x80] * 16)
    want += [-0.25 * -8] * 16 + [0.0] * 16
    # block 2: d = 3 * 2^-24 (subnormal), byte j = 0xF0 | (j & 0xF)
    qs = [0xF0 | j for j in range(16)]
    blocks += _h(0x0003) + bytes(qs)
    want += [3 * 2.0 ** -24 * (j - 8) for j in range(16)] + [3 * 2.0 ** -24 * 7] * 16
    return np.frombuffer(blocks, np.uint8).copy(), np.array(want, np.float64)


def test_scale_bit_patterns_decode_as_written():
    for bits, v in SCALES.items():
        assert float(np.frombuffer(_h(bits), np.float16)[0]) == v


@pytest.mark.parametrize("qtype,kat", [(Q8_0, q8_kat), (Q4_0, q4_kat)])
def test_oracle_dequantises_the_known_answer_blocks(qtype, kat):
    blocks, want = kat()
    K = want.size
    got = oracle.dequant_q(qtype, blocks, 1, K)[0].astype(np.float64)
    assert np.array_equal(got, want), np.nonzero(got != want)


@pytest.mark.parametrize("qtype,kat", [(Q8_0, q8_kat), (Q4_0, q4_kat)])
def test_gguf_py_dequantises_the_known_answer_blocks(qtype, kat):
    """The independent implementation agrees with the written-out weights too,
    so the blocks above mean what this file says they mean."""
    blocks, want = kat()
    gt = gguf.GGMLQuantizationType.Q8_0 if qtype == Q8_0 else gguf.GGMLQuantizationType.Q4_0
    got = gguf.quants.dequantize(blocks.reshape(1, -1), gt)[0].astype(np.float64)
    assert np.array_equal(got, want)


def test_gguf_py_version():
    import importlib.metadata as md

    assert md.version("gguf") == GGUF_PY_VERSION


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0])
@pytest.mark.parametrize("N,K", [(1, 32), (7, 256), (33, 4096)])
def test_oracle_matches_gguf_py_on_its_own_quantised_weights(qtype, N, K):
    """gguf-py quantises a random matrix; the oracle dequantises its bytes bit for
    bit like gguf-py does."""
    rng = np.random.default_rng(N * K + qtype)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W[0, :32] = 0.0
    gt = gguf.GGMLQuantizationType.Q8_0 if qtype == Q8_0 else gguf.GGMLQuantizationType.Q4_0
    blocks = gguf.quants.quantize(W, gt)
    want = gguf.quants.dequantize(blocks, gt).astype(np.float32)
    got = oracle.dequant_q(qtype, blocks.reshape(-1), N, K)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0])
def test_oracle_matches_gguf_py_on_arbitrary_bytes(qtype):
    """Random payload bytes with random finite scales (subnormal to maximal)."""
    rng = np.random.default_rng(99 + qtype)
    bb = 34 if qtype == Q8_0 else 18
    N, nblk = 16, 8
    b = rng.integers(0, 256, (N, nblk, bb), dtype=np.uint8)
    d = np.concatenate([rng.standard_normal(N * nblk // 2) * 1e-2,
                        rng.uniform(-1, 1, N * nblk // 4) * 6e-8,
                        rng.choice([-65504.0, 65504.0, 0.0], N * nblk // 4)]).astype(np.float16)
    b[..., 0:2] = d.view(np.uint8).reshape(N, nblk, 2)
    gt = gguf.GGMLQuantizationType.Q8_0 if qtype == Q8_0 else gguf.GGMLQuantizationType.Q4_0
    want = gguf.quants.dequantize(b.reshape(N, nblk * bb), gt).astype(np.float32)
    got = oracle.dequant_q(qtype, b.reshape(-1), N, 32 * nblk)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------ GGUF files

def test_reader_reads_a_file_written_by_gguf_py(pkg, tmp_path):
    from bmle_b200 import gguf as rd

    rng = np.random.default_rng(5)
    path = tmp_path / "gguf_py.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_uint32("llama.block_count", 32)
    w.add_uint64("llama.context_length", 8192)
    w.add_float32("llama.rope.freq_base", 500000.0)
    w.add_float64("t.f64", 1e-5)
    w.add_int32("t.i32", -7)
    w.add_bool("t.bool", True)
    w.add_string("general.name", "gguf-py pin")
    w.add_array("t.arr", [1, 2, 3])
    W16 = (rng.standard_normal((24, 64)) * 0.02).astype(np.float16)   # [N, K]
    W32 = rng.standard_normal((3, 8)).astype(np.float32)
    Wq = (rng.standard_normal((4, 64)) * 0.02).astype(np.float32)
    q8 = gguf.quants.quantize(Wq, gguf.GGMLQuantizationType.Q8_0)
    q4 = gguf.quants.quantize(Wq, gguf.GGMLQuantizationType.Q4_0)
    w.add_tensor("blk.0.attn_q.weight", W16)
    w.add_tensor("norm.weight", W32)
    w.add_tensor("blk.0.ffn_down.weight", q8, raw_shape=q8.shape,
                 raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    w.add_tensor("blk.0.ffn_up.weight", q4, raw_shape=q4.shape,
                 raw_dtype=gguf.GGMLQuantizationType.Q4_0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    ref = gguf.GGUFReader(str(path))
    with rd.GGUFFile(path) as f:
        assert f.version == 3 and f.alignment == 32
        md = f.metadata()
        assert md["general.architecture"] == "llama"
        assert md["llama.block_count"] == 32 and md["llama.context_length"] == 8192
        assert md["llama.rope.freq_base"] == 500000.0 and md["t.f64"] == 1e-5
        assert md["t.i32"] == -7 and md["t.bool"] == 1
        assert md["general.name"] == "gguf-py pin"
        assert md["t.arr"][0] == "array" and md["t.arr"][2] == 3
        assert [t.name for t in f.tensors] == [t.name for t in ref.tensors]
        for t, r in zip(f.tensors, ref.tensors):
            assert t.type == int(r.tensor_type)
            assert t.dims == tuple(int(x) for x in r.shape)
            assert t.offset == int(r.data_offset)
            assert t.nbytes == int(r.n_bytes)
            assert np.array_equal(f.data(t.name), np.asarray(r.data).reshape(-1).view(np.uint8))
        assert f.tensor("blk.0.attn_q.weight").shape == (24, 64)
        assert np.array_equal(f.data("blk.0.attn_q.weight").view(np.float16).reshape(24, 64), W16)
        assert np.array_equal(f.data("blk.0.ffn_down.weight"), q8.reshape(-1))
        assert np.array_equal(f.data("blk.0.ffn_up.weight"), q4.reshape(-1))


def _gguf_string(s: bytes) -> bytes:
    return struct.pack("<Q", len(s)) + s  # gguf_string_t: uint64 len, then the bytes


def spec_file() -> tuple[bytes, dict]:
    """A GGUF v3 file assembled field by field from the published layout (not by
    tests/gguf_writer.py): returns the bytes and what a reader must find."""
    q8, q8w = q8_kat()   # one row, K = 128: 4 blocks = 136 bytes
    q4, q4w = q4_kat()   # one row, K = 96: 3 blocks = 54 bytes
    f16 = np.array([[1.0, -2.0, 0.5, 65504.0]], np.float16)  # [N=1, K=4]
    out = b"GGUF"                                 # magic, 4 bytes
    out += struct.pack("<I", 3)                   # version: uint32
    out += struct.pack("<Q", 3)                   # tensor_count: uint64
    out += struct.pack("<Q", 3)                   # metadata_kv_count: uint64
    # metadata: key (gguf_string), value type (uint32), value
    out += _gguf_string(b"general.architecture") + struct.pack("<I", 8) + _gguf_string(b"llama")
    out += _gguf_string(b"general.alignment") + struct.pack("<I", 4) + struct.pack("<I", 64)
    out += _gguf_string(b"llama.block_count") + struct.pack("<I", 4) + struct.pack("<I", 2)
    # tensor infos: name, n_dims (uint32), dims (uint64 each, innermost first),
    # ggml type (uint32), offset from the start of the data section (uint64,
    # a multiple of the alignment)
    out += _gguf_string(b"w.q8") + struct.pack("<I", 2) + struct.pack("<QQ", 128, 1)
    out += struct.pack("<I", GGML_Q8_0) + struct.pack("<Q", 0)
    out += _gguf_string(b"w.q4") + struct.pack("<I", 2) + struct.pack("<QQ", 96, 1)
    out += struct.pack("<I", GGML_Q4_0) + struct.pack("<Q", 192)   # 136 rounded up to 64
    out += _gguf_string(b"w.f16") + struct.pack("<I", 2) + struct.pack("<QQ", 4, 1)
    out += struct.pack("<I", 1) + struct.pack("<Q", 256)           # 192 + 54 rounded up
    data_start = (len(out) + 63) // 64 * 64      # the data section starts aligned
    out += b"\0" * (data_start - len(out))
    out += q8.tobytes() + b"\0" * (192 - 136)
    out += q4.tobytes() + b"\0" * (256 - 192 - 54)
    out += f16.tobytes()
    return out, {"data_start": data_start, "q8": (q8, q8w), "q4": (q4, q4w), "f16": f16}


def test_reader_reads_the_spec_assembled_file(pkg, tmp_path):
    from bmle_b200 import gguf as rd

    raw, want = spec_file()
    path = tmp_path / "spec.gguf"
    path.write_bytes(raw)
    ds = want["data_start"]
    with rd.GGUFFile(path) as f:
        assert f.version == 3 and f.alignment == 64
        assert f.meta("general.architecture") == "llama" and f.meta("llama.block_count") == 2
        t = {x.name: x for x in f.tensors}
        assert [x.name for x in f.tensors] == ["w.q8", "w.q4", "w.f16"]
        assert (t["w.q8"].type, t["w.q8"].dims, t["w.q8"].offset, t["w.q8"].nbytes) == \
            (GGML_Q8_0, (128, 1), ds, 136)
        assert (t["w.q4"].type, t["w.q4"].dims, t["w.q4"].offset, t["w.q4"].nbytes) == \
            (GGML_Q4_0, (96, 1), ds + 192, 54)
        assert (t["w.f16"].type, t["w.f16"].dims, t["w.f16"].offset, t["w.f16"].nbytes) == \
            (1, (4, 1), ds + 256, 8)
        assert np.array_equal(f.data("w.q8"), want["q8"][0])
        assert np.array_equal(f.data("w.q4"), want["q4"][0])
        assert np.array_equal(f.data("w.f16").view(np.float16), want["f16"].reshape(-1))
        # the blocks the reader hands out dequantise to the written-out weights
        got = oracle.dequant_q(Q8_0, f.data("w.q8"), 1, 128)[0].astype(np.float64)
        assert np.array_equal(got, want["q8"][1])
    # gguf-py reads the same file the same way
    r = gguf.GGUFReader(str(path))
    assert [x.name for x in r.tensors] == ["w.q8", "w.q4", "w.f16"]
    assert [int(x.data_offset) for x in r.tensors] == [ds, ds + 192, ds + 256]


# ------------------------------------------------------------------ GPU

@pytest.mark.gpu
@pytest.mark.parametrize("qtype,kat", [(Q8_0, q8_kat), (Q4_0, q4_kat)])
def test_cuda_repack_and_gemv_reproduce_the_known_answers(pkg, dev, qtype, kat):
    """Through the product path (engine_cuda_quant_repack + engine_cuda_gemv_q_nk):
    with one-hot activations x = e_j the output is row n's weight j, exact in
    FP16 for these blocks, so every weight (nibble order included) is read back
    against the written-out answer."""
    import torch

    blocks, want = kat()
    K = want.size
    N = 2  # two rows: the KAT row and its negation (scales flipped)
    b2 = blocks.reshape(K // 32, -1).copy()
    neg = b2.copy()
    neg[:, 0:2] = (-b2[:, 0:2].copy().view(np.float16)).view(np.uint8)
    rows = np.concatenate([b2.reshape(-1), neg.reshape(-1)])
    q, sc = pkg.ops.quant_repack(qtype, torch.from_numpy(rows).to(dev), N, K)
    got = np.empty((N, K), np.float64)
    for j in range(K):
        x = torch.zeros(K, device=dev, dtype=torch.float16)
        x[j] = 1.0
        got[:, j] = pkg.ops.gemv_q(qtype, q, sc, x).float().cpu().numpy()
    assert np.array_equal(got[0], want), np.nonzero(got[0] != want)
    assert np.array_equal(got[1], -want)


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [Q8_0, Q4_0])
def test_cuda_gemv_on_gguf_py_quantised_weights(pkg, dev, qtype):
    """Weights quantised by gguf-py (not by this repository), through the CUDA
    repack + GEMV, against the FP64 oracle under the CUDA-core GEMV bound."""
    import torch

    from tests import bounds

    N, K = 512, 4096
    rng = np.random.default_rng(3 + qtype)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    gt = gguf.GGMLQuantizationType.Q8_0 if qtype == Q8_0 else gguf.GGMLQuantizationType.Q4_0
    blocks = gguf.quants.quantize(W, gt).reshape(-1)
    x = rng.standard_normal(K).astype(np.float16)
    q, sc = pkg.ops.quant_repack(qtype, torch.from_numpy(blocks).to(dev), N, K)
    y = pkg.ops.gemv_q(qtype, q, sc, torch.from_numpy(x).to(dev)).float().cpu().numpy()
    _, exact = oracle.gemv_q(qtype, blocks, x, want_f32=True)
    wdq = gguf.quants.dequantize(blocks.reshape(N, -1), gt).astype(np.float64)
    absdot = np.abs(wdq) @ np.abs(x.astype(np.float64))
    bounds.check(y.astype(np.float64), exact.astype(np.float64),
                 bounds.gemv16_bound(K, absdot, exact), f"gemv_q{qtype} on gguf-py blocks")
