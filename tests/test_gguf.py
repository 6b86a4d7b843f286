"""The library's GGUF reader (host code, no GPU) against the reference's own
parse_gguf_tensors and load_tokenizer_tokens (qwen_server.c:113-266, compiled
from its sources into oracle/_ref), on files written by tests/gguf_writer.py."""
import struct

import numpy as np
import pytest

import gguf_writer as gw


def _file(tmp_path, name="m.gguf", alignment=32, honour=True, extra_meta=()):
    rng = np.random.default_rng(7)
    meta = [("general.architecture", gw.STR, "qwen2"),
            ("qwen2.block_count", gw.U32, 28),
            ("general.file_type", gw.U32, 2),
            ("a.u8", gw.U8, 200), ("a.i8", gw.I8, -5), ("a.u16", gw.U16, 60000),
            ("a.i16", gw.I16, -30000), ("a.i32", gw.I32, -7), ("a.f32", gw.F32, 1.5),
            ("a.bool", gw.BOOL, True), ("a.u64", gw.U64, 1 << 40), ("a.i64", gw.I64, -(1 << 40)),
            ("a.f64", gw.F64, 2.25), ("a.str", gw.STR, "héllo"),
            ("a.arr_u32", gw.ARR, (gw.U32, [1, 2, 3])),
            ("a.arr_f64", gw.ARR, (gw.F64, [0.5, 1.5])),
            ("a.arr_i8", gw.ARR, (gw.I8, [-1, 1, 0])),
            ("tokenizer.ggml.tokens", gw.ARR, (gw.STR, ["a", "Ġb", "ĊĠ", "", "<|im_end|>"] +
                                               [f"x{i}" for i in range(45)])),
            ("tokenizer.ggml.token_type", gw.ARR, (gw.I32, [1] * 50)),
            *extra_meta]
    tensors = [("token_embd.weight", gw.T_Q4_0, [64, 50], rng.integers(0, 256, 50 * 36, np.uint8)),
               ("output_norm.weight", gw.T_F32, [64], rng.standard_normal(64).astype(np.float32)),
               ("output.weight", gw.T_Q6_K, [256, 50], rng.integers(0, 256, 50 * 210, np.uint8)),
               ("blk.0.attn_q.bias", gw.T_F32, [7], rng.standard_normal(7).astype(np.float32)),
               ("blk.0.f16", gw.T_F16, [3, 5, 2], rng.integers(0, 256, 60, np.uint8)),
               ("blk.0.q8", gw.T_Q8_0, [32, 3], rng.integers(0, 256, 3 * 34, np.uint8))]
    path = tmp_path / name
    offsets = gw.write(path, meta, tensors, alignment=alignment, honour_alignment_key=honour)
    return path, tensors, offsets


def test_reader_matches_reference_parser(pkg, orc, tmp_path):
    if not orc.have_reference():
        pytest.skip("oracle/_ref not built")
    path, tensors, offsets = _file(tmp_path)
    ref, ref_start = orc.ref_gguf_parse(str(path))
    with pkg.Gguf(str(path)) as g:
        ours = g.tensors()
        assert [t["name"] for t in ours] == [t["name"] for t in ref]
        for a, b in zip(ours, ref):
            assert (a["n_dims"], a["ne"], a["type"], a["offset"]) == \
                   (b["n_dims"], b["ne"], b["type"], b["offset"])
        assert [t["offset"] for t in ours] == [offsets[n] for n, *_ in tensors]
        assert g.vocab_size() == 50
        for i in (0, 1, 2, 3, 4, 49):
            assert g.token(i) == orc.ref_gguf_token(str(path), i)


def test_reader_values(pkg, tmp_path):
    path, tensors, offsets = _file(tmp_path)
    with pkg.Gguf(str(path)) as g:
        for name, tt, ne, data in tensors:
            assert np.array_equal(g.read(name), np.frombuffer(bytes(data), dtype=np.uint8))
            info = g.find(name)
            assert info["ne"] == ne and info["type"] == tt and info["bytes"] == len(bytes(data))
        assert g.meta_int("qwen2.block_count") == 28
        assert g.meta_int("a.i16") == -30000 and g.meta_int("a.u64") == 1 << 40
        assert g.meta_int("a.bool") == 1 and g.meta_int("a.i8") == -5
        with pytest.raises(pkg.GqaError):
            g.meta_int("a.f32")          # not an integer key
        with pytest.raises(pkg.GqaError):
            g.find("blk.9.attn_q.weight")  # absent: an error, not an exit
        assert g.token(1) == "Ġb".encode() and g.token(3) == b""


def test_reader_honours_alignment(pkg, orc, tmp_path):
    """general.alignment = 64: the data starts on 64 (the reference assumes 32
    and would read other bytes; both agree at the default)."""
    path, tensors, offsets = _file(tmp_path, alignment=64,
                                   extra_meta=[("general.alignment", gw.U32, 64)])
    with pkg.Gguf(str(path)) as g:
        for (name, *_), t in zip(tensors, g.tensors()):
            assert t["offset"] == offsets[name] and t["offset"] % 64 == 0
        assert np.array_equal(g.read("output.weight"),
                              np.frombuffer(bytes(tensors[2][3]), dtype=np.uint8))


def test_damaged_files_are_errors(pkg, tmp_path):
    path, tensors, offsets = _file(tmp_path)
    good = path.read_bytes()
    bad = tmp_path / "bad.gguf"
    cases = [b"GGUX" + good[4:],                                 # magic
             good[:4] + struct.pack("<I", 9) + good[8:],         # version
             good[:8] + struct.pack("<Q", 1 << 50) + good[16:],  # tensor count
             good[:16] + struct.pack("<Q", 1 << 50) + good[24:]]  # key count
    last_end = max(offsets[n] + len(np.ascontiguousarray(d).tobytes()) for n, _, _, d in tensors)
    cases += [good[:n] for n in (0, 3, 10, 24, 40, 100, 400, 900, last_end - 1)]  # truncations
    for i, data in enumerate(cases):
        bad.write_bytes(data)
        with pytest.raises(pkg.GqaError):
            pkg.Gguf(str(bad))
    with pytest.raises(pkg.GqaError):
        pkg.Gguf(str(tmp_path / "missing.gguf"))


def test_qwen_shaped_file(pkg, orc, tmp_path):
    """The Qwen2.5-1.5B tensor names and shapes the loader expects, at two
    layers and a small vocabulary; the reference parser agrees."""
    path = tmp_path / "q.gguf"
    offsets, arrays = gw.qwen_model(path, pkg.seeded, n_layers=2, vocab=300, seed=3)
    with pkg.Gguf(str(path)) as g:
        t = g.find("blk.1.ffn_down.weight")
        assert t["ne"] == [8960, 1536] and t["type"] == gw.T_Q4_0
        assert t["bytes"] == 1536 * 280 * 18 and t["offset"] == offsets["blk.1.ffn_down.weight"]
        assert np.array_equal(g.read("output.weight"), arrays["head"])
        assert g.meta_int("qwen2.block_count") == 2
        if orc.have_reference():
            ref, _ = orc.ref_gguf_parse(str(path))
            assert [(r["name"], r["offset"]) for r in ref] == \
                   [(x["name"], x["offset"]) for x in g.tensors()]


def test_names_are_bytes(pkg, tmp_path):
    """A tensor name that is not UTF-8 (the format says UTF-8; the reference
    reads names as bytes) is listed, found and read by the same name."""
    path = tmp_path / "n.gguf"
    name = b"blk.0.\xff\xfe.weight"
    data = np.arange(4, dtype=np.float32)
    gw.write(path, [("general.architecture", gw.STR, "qwen2")],
             [(name, gw.T_F32, [4], data.tobytes())])
    with pkg.Gguf(str(path)) as g:
        (t,) = g.tensors()
        assert t["name"].encode("utf-8", "surrogateescape") == name
        assert np.array_equal(g.read(t["name"]).view(np.float32), data)


def test_mutated_files_are_read_or_refused(pkg, tmp_path):
    """300 seeded mutations of a small model file -- bytes changed in the
    header, metadata and tensor table, 32-bit fields set to extreme values,
    truncations anywhere: each file is either read or refused with GqaError;
    nothing crashes or reads past the end."""
    path = tmp_path / "m.gguf"
    gw.qwen_model(path, pkg.seeded, n_layers=1, vocab=64, seed=2, model="0.5b")
    good = path.read_bytes()
    rng = np.random.default_rng(2024)
    bad = tmp_path / "bad.gguf"
    refused = 0
    for it in range(300):
        b = bytearray(good)
        if it % 3 == 0:
            for _ in range(int(rng.integers(1, 8))):
                b[int(rng.integers(0, min(len(b), 4096)))] = int(rng.integers(0, 256))
        elif it % 3 == 1:
            i = int(rng.integers(0, min(len(b), 4096) - 4)) & ~3
            v = int(rng.choice([0, 1, 0x7FFFFFFF, 0xFFFFFFFF, 0x80000000]))
            b[i:i + 4] = v.to_bytes(4, "little")
        else:
            b = b[:int(rng.integers(0, len(b)))]
        bad.write_bytes(bytes(b))
        try:
            with pkg.Gguf(str(bad)) as g:
                for t in g.tensors():
                    assert t["offset"] + t["bytes"] <= len(b)
                for i in range(min(g.vocab_size(), 8)):
                    g.token(i)
                try:
                    g.read("output.weight")
                except pkg.GqaError:
                    pass
        except pkg.GqaError:
            refused += 1
    assert refused > 0
