"""CPU: the memory-mapped GGUF reader (csrc/gguf.cpp through gguf.GGUFFile).

Files are written by tests/gguf_writer.py, an independent restatement of the
published GGUF layout.  The reader must return every metadata value, tensor
name, type, dims, offset and byte exactly; and it must turn every malformed or
truncated file into ENGINE_ERR_FORMAT (an EngineError), never a crash or an
out-of-range read: every prefix of a valid file, corrupted fields, absurd
counts and lengths, and random byte flips in the header are all tried.
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

from tests import gguf_writer as gw
from tests import quant_np as qn


def _meta():
    return [
        ("general.architecture", gw.STRING, "llama"),
        ("general.name", gw.STRING, "unit-test"),
        ("llama.block_count", gw.UINT32, 32),
        ("llama.embedding_length", gw.UINT64, 4096),
        ("llama.rope.freq_base", gw.FLOAT32, 500000.0),
        ("llama.attention.layer_norm_rms_epsilon", gw.FLOAT64, 1e-5),
        ("t.u8", gw.UINT8, 250), ("t.i8", gw.INT8, -5), ("t.u16", gw.UINT16, 65000),
        ("t.i16", gw.INT16, -30000), ("t.i32", gw.INT32, -7), ("t.i64", gw.INT64, -(2 ** 40)),
        ("t.bool", gw.BOOL, True),
        ("tokenizer.ggml.tokens", gw.ARRAY, (gw.STRING, ["<s>", "</s>", "hello"])),
        ("tokenizer.ggml.scores", gw.ARRAY, (gw.FLOAT32, [0.0, -1.0, -2.5])),
        ("t.nested", gw.ARRAY, (gw.ARRAY, [(gw.UINT32, [1, 2]), (gw.UINT32, [3])])),
    ]


def _tensors(rng):
    W16 = (rng.standard_normal((64, 32)) * 0.02).astype(np.float16)      # [N=64, K=32]
    W32 = rng.standard_normal((5, 3)).astype(np.float32)
    q8 = qn.quantize(qn.Q8_0, (rng.standard_normal((4, 64)) * 0.02).astype(np.float32))
    q4 = qn.quantize(qn.Q4_0, (rng.standard_normal((3, 96)) * 0.02).astype(np.float32))
    bf = rng.integers(0, 2 ** 16, (2, 8), dtype=np.uint16)
    qk = rng.integers(0, 256, 2 * 144, dtype=np.uint8)                     # Q4_K: 256-blocks
    return [
        ("blk.0.attn_q.weight", gw.F16, (32, 64), W16.tobytes()),
        ("norm.weight", gw.F32, (3, 5), W32.tobytes()),
        ("blk.0.ffn_down.weight", gw.Q8_0, (64, 4), q8.tobytes()),
        ("blk.0.ffn_up.weight", gw.Q4_0, (96, 3), q4.tobytes()),
        ("bf.weight", gw.BF16, (8, 2), bf.tobytes()),
        ("qk.weight", 12, (256, 2), qk.tobytes()),
        ("unknown.weight", 99, (7,), b"\x01" * 7),
    ]


def _write(tmp_path, name, data: bytes):
    p = tmp_path / name
    p.write_bytes(data)
    return p


def _open(pkg, path):
    return pkg.gguf.GGUFFile(path)


@pytest.mark.parametrize("alignment,version", [(32, 3), (64, 3), (32, 2)])
def test_round_trip(pkg, tmp_path, alignment, version):
    rng = np.random.default_rng(alignment + version)
    meta = _meta() + ([("general.alignment", gw.UINT32, alignment)] if alignment != 32 else [])
    tens = _tensors(rng)
    blob, offsets = gw.build(meta, tens, alignment=alignment, version=version)
    path = _write(tmp_path, "m.gguf", blob)
    with _open(pkg, path) as f:
        assert f.version == version and f.alignment == alignment
        md = f.metadata()
        assert md["general.architecture"] == "llama" and md["general.name"] == "unit-test"
        assert md["llama.block_count"] == 32 and md["llama.embedding_length"] == 4096
        assert md["llama.rope.freq_base"] == 500000.0
        assert md["llama.attention.layer_norm_rms_epsilon"] == 1e-5
        assert (md["t.u8"], md["t.i8"], md["t.u16"], md["t.i16"], md["t.i32"], md["t.i64"],
                md["t.bool"]) == (250, -5, 65000, -30000, -7, -(2 ** 40), 1)
        assert md["tokenizer.ggml.tokens"] == ("array", gw.STRING, 3)
        assert md["tokenizer.ggml.scores"] == ("array", gw.FLOAT32, 3)
        assert md["t.nested"] == ("array", gw.ARRAY, 2)
        assert [t.name for t in f.tensors] == [t[0] for t in tens]
        sizes = {gw.F16: 2, gw.F32: 4, gw.BF16: 2}
        for (name, ty, dims, data), t in zip(tens, f.tensors):
            assert t.type == ty and t.dims == dims and t.offset == offsets[name]
            assert t.offset % alignment == 0
            known = ty != 99
            assert t.nbytes == (len(data) if known else 0)
            if known:
                assert bytes(f.data(name)) == data
            if ty in sizes:
                assert t.nbytes == sizes[ty] * int(np.prod(dims))
        assert f.tensor("blk.0.attn_q.weight").shape == (64, 32)


def test_block_tensors_decode_like_the_oracle(pkg, tmp_path):
    """The mapped Q8_0 / Q4_0 bytes are the blocks quant_np wrote: the oracle
    dequantises them to the same weights."""
    import oracle

    rng = np.random.default_rng(5)
    tens = _tensors(rng)
    blob, _ = gw.build(_meta(), tens)
    with _open(pkg, _write(tmp_path, "b.gguf", blob)) as f:
        for name, qt, (K, N) in (("blk.0.ffn_down.weight", qn.Q8_0, (64, 4)),
                                 ("blk.0.ffn_up.weight", qn.Q4_0, (96, 3))):
            got = oracle.dequant_q(qt, np.array(f.data(name)), N, K)
            want = qn.dequantize(qt, np.frombuffer(dict((t[0], t[3]) for t in tens)[name],
                                                   np.uint8), N, K)
            assert np.array_equal(got, want)


def _expect_format_error(pkg, path):
    with pytest.raises(pkg.EngineError) as ei:
        pkg.gguf.GGUFFile(path)
    assert ei.value.code == pkg.gguf.ERR_FORMAT, str(ei.value)
    return str(ei.value)


def test_every_truncation_is_a_format_error(pkg, tmp_path):
    """Each prefix that cuts into the header, metadata, tensor table or any
    sized tensor's data is rejected; a cut only in the final padding, or in the
    data of a type the reader cannot size, still reads."""
    rng = np.random.default_rng(11)
    tens = _tensors(rng)
    blob, offsets = gw.build(_meta(), tens)
    data_end = max(offsets[n] + len(d) for n, ty, _, d in tens if ty != 99)
    for cut in list(range(0, 200)) + list(range(200, len(blob), 7)):
        path = _write(tmp_path, "t.gguf", blob[:cut])
        if cut >= data_end:
            with _open(pkg, path) as f:
                assert len(f.tensors) == len(tens)
        else:
            _expect_format_error(pkg, path)


def _patch(blob: bytes, at: int, fmt: str, value) -> bytes:
    b = bytearray(blob)
    struct.pack_into(fmt, b, at, value)
    return bytes(b)


def test_corrupted_fields_are_format_errors(pkg, tmp_path):
    tens = [("w", gw.F16, (32, 2), b"\0" * 128)]
    good, _ = gw.build([("k", gw.UINT32, 1)], tens)
    ok = _write(tmp_path, "ok.gguf", good)
    with _open(pkg, ok) as f:
        assert f.tensors[0].nbytes == 128
    # header fields: magic, version, absurd counts
    assert "magic" in _expect_format_error(pkg, _write(tmp_path, "a", b"GGUX" + good[4:]))
    for v in (1, 4):
        assert "version" in _expect_format_error(pkg, _write(tmp_path, "b", _patch(good, 4, "<I", v)))
    assert "count" in _expect_format_error(pkg, _write(tmp_path, "c", _patch(good, 8, "<Q", 2 ** 40)))
    assert "count" in _expect_format_error(pkg, _write(tmp_path, "d", _patch(good, 16, "<Q", 2 ** 62)))
    # the metadata key length (right after the 24-byte header)
    _expect_format_error(pkg, _write(tmp_path, "e", _patch(good, 24, "<Q", 2 ** 63)))
    # unknown value type
    kv_type_at = 24 + 8 + 1
    assert "value type" in _expect_format_error(pkg, _write(tmp_path, "f", _patch(good, kv_type_at, "<I", 77)))
    # tensor table: n_dims, a misaligned offset, an offset past the end
    t_at = kv_type_at + 4 + 4 + 8 + 1          # name length, then "w"
    assert "dims" in _expect_format_error(pkg, _write(tmp_path, "g", _patch(good, t_at, "<I", 5)))
    off_at = t_at + 4 + 16 + 4
    assert "alignment" in _expect_format_error(pkg, _write(tmp_path, "h", _patch(good, off_at, "<Q", 8)))
    assert "end of the file" in _expect_format_error(pkg, _write(tmp_path, "i", _patch(good, off_at, "<Q", 4096)))
    # a block type whose row is not whole blocks
    bad, _ = gw.build([], [("q", gw.Q8_0, (48, 1), b"\0" * 51)])
    assert "block" in _expect_format_error(pkg, _write(tmp_path, "j", bad))
    # duplicates and a bad alignment
    dup, _ = gw.build([], [("w", gw.F16, (8,), b"\0" * 16), ("w", gw.F16, (8,), b"\0" * 16)])
    assert "duplicate" in _expect_format_error(pkg, _write(tmp_path, "k", dup))
    dupk, _ = gw.build([("k", gw.UINT8, 1), ("k", gw.UINT8, 2)], [])
    assert "duplicate" in _expect_format_error(pkg, _write(tmp_path, "l", dupk))
    al, _ = gw.build([("general.alignment", gw.UINT32, 48)], [])
    assert "alignment" in _expect_format_error(pkg, _write(tmp_path, "m", al))
    # an empty and a missing file
    _expect_format_error(pkg, _write(tmp_path, "n", b""))
    with pytest.raises(pkg.EngineError) as ei:
        pkg.gguf.GGUFFile(tmp_path / "does-not-exist.gguf")
    assert ei.value.code == pkg.gguf.ERR_IO


def test_random_header_corruption_never_crashes(pkg, tmp_path):
    """Flipped bytes anywhere before the tensor data either still parse or are
    a format error; the process survives every one."""
    rng = np.random.default_rng(3)
    blob, offsets = gw.build(_meta(), _tensors(rng))
    head = min(offsets.values())
    for _ in range(400):
        b = bytearray(blob)
        for _ in range(int(rng.integers(1, 4))):
            b[int(rng.integers(0, head))] = int(rng.integers(0, 256))
        path = _write(tmp_path, "r.gguf", bytes(b))
        try:
            f = pkg.gguf.GGUFFile(path)
            f.metadata()
            for t in f.tensors:
                f.data(t.name)
            f.close()
        except pkg.EngineError as e:
            assert e.code == pkg.gguf.ERR_FORMAT, str(e)


def test_lookups(pkg, tmp_path):
    blob, _ = gw.build(_meta(), _tensors(np.random.default_rng(1)))
    with _open(pkg, _write(tmp_path, "l.gguf", blob)) as f:
        with pytest.raises(pkg.EngineError, match="no tensor"):
            f.tensor("missing.weight")
        with pytest.raises(pkg.EngineError, match="no key"):
            f.meta("missing.key")
        assert f.meta("general.name") == "unit-test"
        h = f._h
        import ctypes
        v = ctypes.c_int64()
        assert pkg.lib().engine_gguf_meta_int(h, b"general.name", ctypes.byref(v)) == 1  # not an int
        d = ctypes.c_double()
        assert pkg.lib().engine_gguf_meta_float(h, b"llama.block_count", ctypes.byref(d)) == 1
        assert pkg.gguf.gemv_qtype(pkg.gguf.Q8_0) == 8 and pkg.gguf.gemv_qtype(pkg.gguf.Q4_0) == 4


# ------------------------------------------------ property-based round trips
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

_INT_RANGES = {gw.UINT8: (0, 255), gw.INT8: (-128, 127), gw.UINT16: (0, 65535),
               gw.INT16: (-32768, 32767), gw.UINT32: (0, 2 ** 32 - 1),
               gw.INT32: (-2 ** 31, 2 ** 31 - 1), gw.UINT64: (0, 2 ** 63 - 1),
               gw.INT64: (-2 ** 63, 2 ** 63 - 1)}


def _scalar(vt):
    if vt in _INT_RANGES:
        lo, hi = _INT_RANGES[vt]
        return st.integers(lo, hi)
    if vt == gw.BOOL:
        return st.booleans()
    if vt == gw.FLOAT32:
        return st.floats(width=32, allow_nan=False)
    if vt == gw.FLOAT64:
        return st.floats(allow_nan=False)
    return st.text(max_size=12)  # STRING


_SCALARS = sorted(_INT_RANGES) + [gw.BOOL, gw.FLOAT32, gw.FLOAT64, gw.STRING]


@st.composite
def _entry(draw, key):
    if draw(st.integers(0, 3)) == 0:  # an array, sometimes of arrays
        et = draw(st.sampled_from(_SCALARS + [gw.ARRAY]))
        if et == gw.ARRAY:
            inner = draw(st.sampled_from(_SCALARS))
            items = draw(st.lists(st.lists(_scalar(inner), max_size=3).map(lambda x: (inner, x)),
                                  max_size=3))
        else:
            items = draw(st.lists(_scalar(et), max_size=4))
        return key, gw.ARRAY, (et, items)
    vt = draw(st.sampled_from(_SCALARS))
    return key, vt, draw(_scalar(vt))


@st.composite
def _model(draw):
    keys = draw(st.lists(st.text("abcdefghij._", min_size=1, max_size=16), unique=True,
                         max_size=8))
    meta = [draw(_entry(k)) for k in keys]
    names = draw(st.lists(st.text("abcdefghij.", min_size=1, max_size=12), unique=True,
                          max_size=5))
    tensors = []
    for n in names:
        ty = draw(st.sampled_from([gw.F32, gw.F16, gw.BF16, gw.Q8_0, gw.Q4_0]))
        block, size = {gw.F32: (1, 4), gw.F16: (1, 2), gw.BF16: (1, 2), gw.Q8_0: (32, 34),
                       gw.Q4_0: (32, 18)}[ty]
        dims = tuple([block * draw(st.integers(1, 3))] +
                     [draw(st.integers(1, 3)) for _ in range(draw(st.integers(0, 3)))])
        nbytes = int(np.prod(dims)) // block * size
        tensors.append((n, ty, dims, draw(st.binary(min_size=nbytes, max_size=nbytes))))
    alignment = draw(st.sampled_from([8, 16, 32, 64, 256]))
    version = draw(st.sampled_from([2, 3]))
    return meta, tensors, alignment, version


@settings(max_examples=150, deadline=None,
          suppress_health_check=[HealthCheck.function_scoped_fixture, HealthCheck.too_slow])
@given(m=_model())
def test_round_trip_property(pkg, tmp_path, m):
    meta, tensors, alignment, version = m
    # (random keys use letters that cannot spell "general.alignment")
    meta = list(meta) + ([("general.alignment", gw.UINT32, alignment)] if alignment != 32 else [])
    blob, offsets = gw.build(meta, tensors, alignment=alignment, version=version)
    path = _write(tmp_path, "p.gguf", blob)
    with _open(pkg, path) as f:
        assert f.version == version and f.alignment == alignment
        md = f.metadata()
        assert list(md) == [k for k, _, _ in meta]
        for k, vt, v in meta:
            if vt == gw.ARRAY:
                assert md[k] == ("array", v[0], len(v[1]))
            elif vt == gw.FLOAT32:
                assert md[k] == float(np.float32(v))
            else:
                assert md[k] == (int(v) if vt == gw.BOOL else v)
        assert [t.name for t in f.tensors] == [t[0] for t in tensors]
        for (n, ty, dims, data), t in zip(tensors, f.tensors):
            assert (t.type, t.dims, t.offset, t.nbytes) == (ty, dims, offsets[n], len(data))
            assert bytes(f.data(n)) == data
