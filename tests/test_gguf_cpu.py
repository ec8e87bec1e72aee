"""GGUF file reading (GgufFile::parse, rce-ingest-gguf/src/parser.rs:446-553)
and the tensor byte ranges QuantWeight::from_gguf uses
(rce-op-qmm/src/lib.rs:173-209), on files written by gguf.build_gguf in the
layout of the reference's own test builder (parser.rs:625-695).  Mirrors the
reference's parser tests: minimal header, string / u32 / array metadata,
tensor infos, several tensors, and its error cases."""
import struct

import numpy as np
import pytest

from rce_b200 import gguf as G
from rce_b200 import synth


def test_minimal_header():
    f = G.GgufFile.parse(G.build_gguf([], []))
    assert f.version == 3 and f.metadata == {} and f.tensors == [] and f.alignment == 32
    assert f.data_offset % 32 == 0


def test_metadata_of_every_type_round_trips():
    meta = [("u8", G.T_U8, 200), ("i8", G.T_I8, -5), ("u16", G.T_U16, 60000), ("i16", G.T_I16, -30000),
            ("u32", G.T_U32, 4_000_000_000), ("i32", G.T_I32, -2_000_000_000), ("f32", G.T_F32, 1.5),
            ("b", G.T_BOOL, True), ("s", G.T_STRING, "llama·3"), ("u64", G.T_U64, 2 ** 40),
            ("i64", G.T_I64, -(2 ** 40)), ("f64", G.T_F64, 0.1),
            ("arr", G.T_ARRAY, (G.T_U32, [1, 2, 3])), ("strs", G.T_ARRAY, (G.T_STRING, ["a", "bc"])),
            ("nested", G.T_ARRAY, (G.T_ARRAY, [(G.T_I8, [1, -1]), (G.T_I8, [])]))]
    f = G.GgufFile.parse(G.build_gguf(meta, []))
    want = {k: v for k, _, v in meta}
    want["arr"], want["strs"], want["nested"] = [1, 2, 3], ["a", "bc"], [[1, -1], []]
    assert f.metadata == want


def test_model_header_accessors():
    meta = [("general.architecture", G.T_STRING, "llama"), ("general.name", G.T_STRING, "tiny"),
            ("llama.block_count", G.T_U32, 22), ("llama.embedding_length", G.T_U32, 2048)]
    f = G.GgufFile.parse(G.build_gguf(meta, []))
    assert f.architecture() == "llama" and f.block_count() == 22 and f.get("llama.embedding_length") == 2048


@pytest.mark.parametrize("align", [32, 64, 4096])
def test_tensors_and_alignment(align):
    rng = np.random.default_rng(align)
    q4k = synth.weights(G.GgufDtype.Q4K, 48, 512, rng)
    q8 = synth.weights(G.GgufDtype.Q8_0, 3, 64, rng)
    q40 = synth.weights(G.GgufDtype.Q4_0, 5, 96, rng)
    q6k = rng.integers(0, 256, G.tensor_byte_size(G.GgufDtype.Q6K, 256 * 4), dtype=np.uint8)
    tensors = [("blk.0.ffn_up.weight", [512, 48], 12, q4k), ("tok_embd", [64, 3], 8, q8),
               ("blk.0.attn_v.weight", [96, 5], 2, q40), ("output.weight", [256, 4], 14, q6k)]
    b = G.build_gguf([("general.architecture", G.T_STRING, "llama")], tensors, alignment=align)
    f = G.GgufFile.parse(b)
    assert f.alignment == align and f.data_offset % align == 0
    assert [t.name for t in f.tensors] == [t[0] for t in tensors]
    for (name, dims, tag, data), t in zip(tensors, f.tensors):
        assert t.dims == dims and t.dtype_tag == tag and t.offset % align == 0
        assert t.numel == int(np.prod(dims)) and t.nbytes == len(data)
        assert bytes(f.tensor_bytes(t)) == bytes(data)
    assert f.tensor("missing") is None


def test_open_maps_the_file(tmp_path):
    rng = np.random.default_rng(1)
    w = synth.weights(G.GgufDtype.Q4K, 32, 256, rng)
    p = tmp_path / "m.gguf"
    p.write_bytes(G.build_gguf([], [("w", [256, 32], 12, w)]))
    f = G.GgufFile.open(p)
    t = f.tensor("w")
    assert np.array_equal(np.frombuffer(f.tensor_bytes(t), np.uint8), w)


def test_version_2_is_accepted():
    f = G.GgufFile.parse(G.build_gguf([], [], version=2))
    assert f.version == 2


@pytest.mark.parametrize("case", ["magic", "version1", "version4", "dims", "truncated", "utf8", "type", "oob"])
def test_malformed_files_are_errors(case):
    good = G.build_gguf([("k", G.T_STRING, "v")], [("w", [32, 1], 8, bytes(34))])
    if case == "magic":
        b = b"GGUX" + good[4:]
    elif case == "version1":
        b = good[:4] + struct.pack("<I", 1) + good[8:]
    elif case == "version4":
        b = good[:4] + struct.pack("<I", 4) + good[8:]
    elif case == "dims":
        b = G.build_gguf([], [("w", [1] * 9, 0, bytes(4))])
    elif case == "truncated":
        b = good[:30]
    elif case == "utf8":
        b = G.build_gguf([("k", G.T_STRING, "v")], [])
        i = b.index(b"k")
        b = b[:i] + b"\xff" + b[i + 1:]
    elif case == "type":
        b = G.build_gguf([("k", G.T_U32, 1)], [])
        i = b.index(b"k") + 1
        b = b[:i] + struct.pack("<I", 99) + b[i + 4:]
    else:
        b = good[:-10]  # the tensor's bytes run past the end of the file
    with pytest.raises(G.GgufParseError):
        f = G.GgufFile.parse(b)
        f.tensor_bytes(f.tensors[0])
