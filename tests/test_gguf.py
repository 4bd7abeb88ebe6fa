"""GGUF reader (planejaja_b200/gguf.py) on CPU.

Files written by gguf-py 0.19.0 (third-party writer, the format's own
tooling) and by the reader's minimal writer are parsed; tensor bytes, shapes,
types, metadata and the data-section alignment must come back exactly.  The
reference loader's sizing bugs (nodestor-formats/src/gguf.rs:268-304: no
Q4_K/Q6_K, Q8_0 at 36 bytes per 32, id 9 read as Q8_0, 32-byte data start
whatever general.alignment says) are checked against the fixed table.
"""
import numpy as np
import pytest

from planejaja_b200 import gguf as G
from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, fmt

gguf_py = pytest.importorskip("gguf")


def _write_with_gguf_py(path, alignment=None):
    from gguf import GGMLQuantizationType as T
    from gguf import GGUFWriter
    w = GGUFWriter(str(path), "llama")
    w.add_name("tiny")
    w.add_uint32("tiny.block_count", 2)
    w.add_float32("tiny.rope.freq_base", 10000.0)
    w.add_array("tiny.list", [1, 2, 3, 4, 5])
    if alignment:
        w.add_custom_alignment(alignment)
    rng = np.random.default_rng(0)
    tens = {}
    f32 = rng.standard_normal((3, 5)).astype(np.float32)
    w.add_tensor("f32", f32)
    tens["f32"] = (f32.tobytes(), (5, 3), 0)
    for name, tid, n, k in (("q4k", Q4_K, 6, 512), ("q6k", Q6_K, 4, 256), ("q8", Q8_0, 5, 64), ("q40", Q4_0, 3, 96),
                            ("q5k", Q5_K, 2, 768)):
        raw = Q.synthetic_weights(n, k, tid, seed=n + k)
        qt = {Q4_K: T.Q4_K, Q5_K: T.Q5_K, Q6_K: T.Q6_K, Q8_0: T.Q8_0, Q4_0: T.Q4_0}[tid]
        rb = fmt(tid).row_bytes(k)
        w.add_tensor(name, raw.reshape(n, rb), raw_dtype=qt)
        tens[name] = (raw.tobytes(), (k, n), tid)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tens


@pytest.mark.parametrize("alignment", [None, 64])
def test_reads_gguf_py_files(tmp_path, alignment):
    path = tmp_path / "tiny.gguf"
    tens = _write_with_gguf_py(path, alignment)
    with G.open_gguf(str(path)) as f:
        assert f.version == 3
        assert f.alignment == (alignment or 32)
        assert f.data_offset % f.alignment == 0
        assert f.metadata["general.name"] == "tiny"
        assert f.metadata["general.architecture"] == "llama"
        assert f.metadata["tiny.block_count"] == 2
        assert f.metadata["tiny.list"] == [1, 2, 3, 4, 5]
        assert abs(f.metadata["tiny.rope.freq_base"] - 10000.0) < 1e-3
        assert set(f.tensors) == set(tens)
        for name, (raw, shape, tid) in tens.items():
            t = f.tensors[name]
            assert t.shape == shape and t.type_id == tid, name
            assert t.offset % f.alignment == 0
            assert bytes(f.data(name)) == raw, name
        assert f.tensors["q4k"].matrix() == (6, 512)
        assert f.tensors["q4k"].matmul_supported and not f.tensors["f32"].matmul_supported


def test_agrees_with_gguf_py_reader(tmp_path):
    from gguf import GGUFReader
    path = tmp_path / "tiny.gguf"
    _write_with_gguf_py(path, 64)
    r = GGUFReader(str(path))
    with G.open_gguf(str(path)) as f:
        for t in r.tensors:
            ours = f.tensors[t.name]
            assert ours.offset == int(t.data_offset)
            assert ours.nbytes == int(t.n_bytes)
            assert ours.type_id == int(t.tensor_type)
            assert list(ours.shape) == [int(d) for d in t.shape]


def test_fixed_sizes_against_reference_table():
    # 4096-weight rows: reference (gguf.rs:288-304) vs ggml
    assert G.tensor_nbytes((4096,), Q8_0) == 128 * 34       # reference: 128 * 36
    assert G.tensor_nbytes((4096,), Q4_K) == 16 * 144       # reference: 4096 * 4 (F32 fallback)
    assert G.tensor_nbytes((4096,), Q6_K) == 16 * 210       # reference: 4096 * 4
    assert G.tensor_nbytes((4096,), Q5_K) == 16 * 176       # reference: 4096 * 4
    assert G.tensor_nbytes((4096,), 9) == 128 * 36          # Q8_1, which the reference reads as Q8_0
    assert G.TYPES[9][0] == "Q8_1"
    with pytest.raises(G.GGUFError):
        G.tensor_nbytes((4096,), 99)  # unknown ids are errors, not F32
    with pytest.raises(G.GGUFError):
        G.tensor_nbytes((100,), Q4_K)  # partial super-block


def test_minimal_writer_round_trip_and_alignment(tmp_path):
    raw = Q.synthetic_weights(3, 256, Q4_K, seed=1)
    for al in (32, 128):
        p = tmp_path / f"m{al}.gguf"
        G.write_minimal(str(p), [("a", (256, 3), Q4_K, raw), ("b", (7,), 0, np.arange(7, dtype=np.float32).tobytes())],
                        {"general.name": "m", "n": 5}, alignment=al)
        with G.open_gguf(str(p)) as f:
            assert f.alignment == al and f.data_offset % al == 0
            assert bytes(f.data("a")) == raw.tobytes()
            assert np.frombuffer(f.data("b"), np.float32).tolist() == list(range(7))
            assert f.metadata["n"] == 5


def test_rejects_malformed_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"NOTGGUF!" + b"\0" * 32)
    with pytest.raises(G.GGUFError):
        G.open_gguf(str(p))
    raw = Q.synthetic_weights(2, 256, Q4_K, seed=2)
    good = tmp_path / "good.gguf"
    G.write_minimal(str(good), [("a", (256, 2), Q4_K, raw)])
    data = good.read_bytes()
    (tmp_path / "short.gguf").write_bytes(data[:-10])  # tensor runs past the end
    with pytest.raises(G.GGUFError):
        G.open_gguf(str(tmp_path / "short.gguf"))
    (tmp_path / "v1.gguf").write_bytes(data[:4] + (1).to_bytes(4, "little") + data[8:])
    with pytest.raises(G.GGUFError):
        G.open_gguf(str(tmp_path / "v1.gguf"))
