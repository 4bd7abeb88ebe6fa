"""NSZ (TCA-TBE) codec on CPU: the oracle pinned on the reference's own file,
the reference's unit tests re-expressed, the package encoder / file writer /
reader against the oracle, and the host tile index's validation."""
import math
import struct

import numpy as np
import pytest

from planejaja_b200 import nsz as Z

STREAMS = {"output_norm.weight": 64, "blk.0.attn_q.weight": 4096, "token_embd.weight": 8192,
           "blk.0.ffn_down.weight": 11008}


@pytest.fixture(scope="module")
def nszg():
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    return dict(np.load(os.path.join(root, "tests", "golden", "nsz_golden.npz")))


def stream(g, name):
    return g["stream_" + name.replace(".", "_")]


def f32(v):
    return np.asarray(v, np.float32)


# ------------------------------------------------- pin: the reference's file
@pytest.mark.parametrize("name", list(STREAMS))
def test_oracle_round_trips_reference_stream(oracle, nszg, name):
    """decode(reference bytes) re-encodes to the same bytes (nsz_convert.rs
    validated these tensors bit-exact when it wrote them)."""
    s, n = stream(nszg, name), STREAMS[name]
    w = oracle.nsz_decode(s, n)
    assert np.array_equal(oracle.nsz_encode(w), s)
    assert np.array_equal(Z.encode(w), s)  # the package encoder too
    # the micro model's weights are N(0, 0.02) (gerador_micro_gguf.py)
    assert np.isfinite(w).all() and abs(float(w.std()) - 0.02) < 0.003 and abs(float(w.mean())) < 0.004
    off = oracle.nsz_offsets(s, n)
    assert np.array_equal(Z.index(s, n), (off // 64).astype(np.uint32))


def test_reference_file_index(nszg):
    hdr, ent = nszg["file_header"].tobytes(), nszg["entries"].tobytes()
    assert hdr[:4] == b"NSZ1"
    version, flags, n, orig, comp = struct.unpack("<HHIQQ", hdr[4:])
    assert (version, flags, n) == (1, 0, 21)
    entries = [Z.Entry.from_bytes(ent[i * 128:(i + 1) * 128]) for i in range(n)]
    assert sum(e.original_size for e in entries) == orig and sum(e.compressed_size for e in entries) == comp
    assert entries[0].compressed_offset == -(-(28 + 21 * 128) // 64) * 64  # data starts 64-aligned
    for a, b in zip(entries, entries[1:]):
        assert b.compressed_offset == a.compressed_offset + a.compressed_size
    by = {e.name: e for e in entries}
    for name, cnt in STREAMS.items():
        e = by[name]
        assert e.dtype == Z.FP32 and e.num_weights == cnt and e.num_tiles == -(-cnt // 512)
        assert e.compressed_size == stream(nszg, name).size
        assert e.to_bytes() == ent[entries.index(e) * 128:(entries.index(e) + 1) * 128]
    assert by["blk.0.ffn_down.weight"].shape == (172, 64, 0, 0)
    assert by["blk.0.ffn_down.weight"].matrix() == (64, 172)
    assert by["token_embd.weight"].matrix() == (128, 64)


def test_writer_reproduces_reference_layout(tmp_path, oracle, nszg):
    """A file written here from the decoded tensors holds the reference's tile bytes."""
    recs = []
    for name, cnt in STREAMS.items():
        recs.append((name, oracle.nsz_decode(stream(nszg, name), cnt), None))
    p = tmp_path / "m.nsz"
    Z.write(str(p), recs)
    with Z.open_nsz(str(p)) as f:
        assert list(f.entries) == list(STREAMS)
        for name, cnt in STREAMS.items():
            assert np.array_equal(f.stream(name), stream(nszg, name))
            assert f.entries[name].num_weights == cnt
            assert f.index(name)[-1] * 64 == f.entries[name].compressed_size


# ------------------------------------------------- reference unit tests
def test_encode_all_same(oracle):  # nsz_encoder.rs:333-347
    t = oracle.nsz_encode_tile(np.ones(512, np.float32))
    assert t[0] == 127 and t[1:3] == b"\0\0" and t[4:6] == b"\0\0"
    assert t[8:72] == b"\xff" * 64


def test_encode_mixed(oracle):  # nsz_encoder.rs:350-361
    w = np.concatenate([np.ones(400), np.full(80, 2.0), np.full(32, 100.0)]).astype(np.float32)
    t = oracle.nsz_encode_tile(w)
    assert t[0] == 127
    assert struct.unpack("<H", t[4:6])[0] == 80 and struct.unpack("<H", t[1:3])[0] == 32


def test_pack_bits_order(oracle):  # nsz_encoder.rs:364-370: bit i of byte i/8, LSB first
    w = np.zeros(512, np.float32)
    w[[0, 2, 3, 7, 8]] = 1.0  # exponent 127 on these, 0 elsewhere: modal 0, these residual
    t = oracle.nsz_encode_tile(w)
    assert t[8] == 0b01110010 and t[9] == 0b11111110  # match bitmap = complement of those bits


def test_compression_ratio_and_tiles(oracle):  # nsz_encoder.rs:373-385, :388-396
    assert len(oracle.nsz_encode_tile(np.full(512, 0.02, np.float32))) < 2048
    s = oracle.nsz_encode(np.ones(1024, np.float32))
    assert oracle.nsz_offsets(s, 1024).size == 3  # 2 tiles


def test_find_modal_first_maximum(oracle):  # nsz_encoder.rs:399-402 and ties
    e = [127, 127, 127, 128, 126, 127, 127]
    w = np.array([math.ldexp(1.0, x - 127) for x in e], np.float32)
    assert oracle.nsz_encode_tile(w)[0] == 127
    w = np.array([4.0, 4.0, 2.0, 2.0], np.float32)  # tie: the smaller exponent wins
    assert oracle.nsz_encode_tile(w)[0] == 128


@pytest.mark.parametrize("case", ["ones", "zeros", "negative", "mixed", "subnormals", "multi", "special"])
def test_reference_round_trips(oracle, case):  # nsz_decoder.rs:240-349
    if case == "ones":
        w = np.ones(512, np.float32)
    elif case == "zeros":
        w = np.zeros(512, np.float32)
    elif case == "negative":
        w = np.full(512, -0.5, np.float32)
    elif case == "mixed":
        w = np.concatenate([0.01 * (np.arange(400) - 200.0) / 200.0, 0.5 * (np.arange(80) - 40.0) / 40.0,
                            100.0 + np.arange(32)]).astype(np.float32)
    elif case == "subnormals":
        w = np.arange(512, dtype=np.uint32).view(np.float32)
    elif case == "multi":
        w = (np.arange(1500) * 0.001 - 0.75).astype(np.float32)
    else:
        w = np.zeros(512, np.float32)
        w[:7] = [np.inf, -np.inf, -0.0, np.finfo(np.float32).tiny, np.finfo(np.float32).max,
                 np.finfo(np.float32).min, np.nan]
    s = oracle.nsz_encode(w)
    d = oracle.nsz_decode(s, w.size)
    assert np.array_equal(d.view(np.uint32), w.view(np.uint32))
    assert np.array_equal(Z.encode(w), s)


def test_file_header_and_entry_round_trip():  # nsz_format.rs:339-374
    e = Z.Entry("blk.0.attn_q.weight", Z.FP32, 16384, 256, 12000, 32, 4096, (64, 64, 0, 0))
    b = e.to_bytes()
    assert len(b) == 128 and Z.Entry.from_bytes(b) == e


# ------------------------------------------------- encoder and decoder, all dtypes
def _weights(rng, dt, n):
    if dt == Z.FP32:
        return (rng.standard_normal(n) * 0.02).astype(np.float32)
    if dt == Z.FP16:
        return (rng.standard_normal(n) * 0.3).astype(np.float16)
    return ((rng.standard_normal(n) * 0.02).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("dt", [Z.FP32, Z.FP16, Z.BF16])
@pytest.mark.parametrize("n", [1, 37, 512, 513, 1500, 4096, 11008])
def test_package_encoder_matches_oracle(oracle, dt, n):
    w = _weights(np.random.default_rng(n + 10 * dt), dt, n)
    s = Z.encode(w, dt)
    assert np.array_equal(s, oracle.nsz_encode(w, dt, reference_quirks=False))
    assert np.array_equal(oracle.nsz_decode(s, n, dt).view(np.uint8), w.view(np.uint8))


def test_fuzz_bit_patterns(oracle):
    """Every exponent, sign and mantissa pattern; wide exponent spread."""
    rng = np.random.default_rng(5)
    w = rng.integers(0, 2 ** 32, 5000, dtype=np.uint64).astype(np.uint32)
    s = Z.encode(w.view(np.float32))
    assert np.array_equal(oracle.nsz_decode(s, w.size).view(np.uint32), w)
    h = rng.integers(0, 2 ** 16, 3000, dtype=np.uint32).astype(np.uint16)
    for dt in (Z.FP16, Z.BF16):
        s = Z.encode(h, dt) if dt == Z.BF16 else Z.encode(h.view(np.float16), dt)
        assert np.array_equal(oracle.nsz_decode(s, h.size, dt), h)


def test_modal_255_quirk(oracle):
    """The reference encoder files exponent 0 as near when the modal exponent
    is 255 and its decoder restores 254; the package encoder keeps it exact."""
    w = np.full(512, np.inf, np.float32)
    w[3] = 1e-40  # exponent 0
    lossy = oracle.nsz_decode(oracle.nsz_encode(w, reference_quirks=True), 512)
    assert (lossy.view(np.uint32)[3] >> 23) == 254
    s = Z.encode(w)
    assert np.array_equal(s, oracle.nsz_encode(w, reference_quirks=False))
    assert np.array_equal(oracle.nsz_decode(s, 512).view(np.uint32), w.view(np.uint32))


# ------------------------------------------------- host index validation
def test_index_rejects_malformed_streams():
    w = (np.random.default_rng(3).standard_normal(1500) * 0.02).astype(np.float32)
    s = Z.encode(w)
    off = Z.index(s, 1500)
    assert off.size == 4 and off[-1] * 64 == s.size
    bad = s.copy()
    bad[3] = 1  # dtype byte
    with pytest.raises(Z.NSZError):
        Z.index(bad, 1500)
    bad = s.copy()
    bad[4] ^= 1  # near count off by one
    with pytest.raises(Z.NSZError):
        Z.index(bad, 1500)
    bad = s.copy()
    bad[8] ^= 0xFF  # match bitmap no longer agrees with the residual count
    with pytest.raises(Z.NSZError):
        Z.index(bad, 1500)
    with pytest.raises(Z.NSZError):
        Z.index(s[:-64], 1500)  # truncated
    with pytest.raises(Z.NSZError):
        Z.index(np.concatenate([s, np.zeros(64, np.uint8)]), 1500)  # trailing bytes
    with pytest.raises(Z.NSZError):
        Z.index(s, 1400)  # wrong weight count
    with pytest.raises(Z.NSZError):
        Z.index(s, 1500, Z.FP16)
    assert Z.index(np.zeros(0, np.uint8), 0).tolist() == [0]


def test_reader_rejects_bad_files(tmp_path):
    p = tmp_path / "x.nsz"
    p.write_bytes(b"GGUF" + b"\0" * 60)
    with pytest.raises(Z.NSZError):
        Z.open_nsz(str(p))
    w = np.ones(600, np.float32)
    Z.write(str(p), [("a", w, None)])
    data = p.read_bytes()
    (tmp_path / "short.nsz").write_bytes(data[:-64])
    with pytest.raises(Z.NSZError):
        Z.open_nsz(str(tmp_path / "short.nsz"))
