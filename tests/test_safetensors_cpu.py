"""The safetensors reader (b2a_safetensors_*, host code, no GPU needed).

The header-validation cases restate the reference's own tests
(test/safetensors.test.js:37-130) on synthetic files built the same way
(u64 length, JSON header, data). The Qwen2.5 tensor inventory is pinned to
the reference's golden/tensor_digest.json (tests/golden/qwen25_tensors.json,
made by tests/golden/make_tensor_inventory.py): the names and shapes the
config implies (config.expectedTensors) must be exactly the real checkpoint's.
"""
import json
import os
import struct

import numpy as np
import pytest

import b2a

HERE = os.path.dirname(os.path.abspath(__file__))


def build(header, data=b""):
    text = json.dumps(header).encode()
    return struct.pack("<Q", len(text)) + text + bytes(data)


OK = {"t": {"dtype": "F32", "shape": [2, 2], "data_offsets": [0, 16]}}


def rejects(image, match):
    with pytest.raises(b2a.B2AError, match=match):
        b2a.Safetensors.fromBytes(image)


def test_opens_a_well_formed_file_and_reports_its_tensors():
    data = np.array([1, 2, 3, 4], np.float32).tobytes()
    st = b2a.Safetensors.fromBytes(build({**OK, "__metadata__": {"format": "pt"}}, data))
    assert st.size == 1
    assert st.names() == ["t"]
    assert st.metadata == {"format": "pt"}
    assert st.info("t").shape == (2, 2)
    assert st.info("t").numel == 4
    assert st.readF32("t").reshape(-1).tolist() == [1, 2, 3, 4]


def test_rejects_a_file_too_short_to_hold_a_header_length():
    rejects(bytes(4), "not a safetensors file")


def test_rejects_a_header_length_that_runs_past_the_end_of_the_file():
    img = bytearray(build(OK, bytes(16)))
    img[:8] = struct.pack("<Q", 1 << 40)
    rejects(bytes(img), "does not fit")


def test_rejects_a_header_that_is_not_json():
    rejects(struct.pack("<Q", 3) + b"{{{", "not valid UTF-8 JSON")


def test_rejects_a_header_that_is_not_utf8():
    rejects(struct.pack("<Q", 4) + b'"\xff"}', "not valid UTF-8 JSON")


def test_rejects_a_header_that_is_not_an_object():
    rejects(struct.pack("<Q", 2) + b"[]", "must be a JSON object")


def test_rejects_an_unknown_dtype_rather_than_guessing_an_element_size():
    rejects(build({"t": {"dtype": "F4_SECRET", "shape": [4], "data_offsets": [0, 16]}}, bytes(16)),
            'unknown dtype "F4_SECRET"')


def test_rejects_a_shape_whose_element_count_disagrees_with_its_byte_range():
    rejects(build({"t": {"dtype": "F32", "shape": [2, 2], "data_offsets": [0, 12]}}, bytes(12)),
            r"shape \[2,2\] of F32 needs 16 bytes but the header reserves 12")


def test_rejects_a_tensor_that_ends_past_the_data_section():
    rejects(build(OK, bytes(8)), "data section is only 8 bytes")


def test_rejects_negative_and_inverted_offsets():
    rejects(build({"t": {"dtype": "F32", "shape": [1], "data_offsets": [8, 4]}}, bytes(16)),
            r"bad data_offsets \[8, 4\]")
    rejects(build({"t": {"dtype": "F32", "shape": [1], "data_offsets": [-4, 0]}}, bytes(16)), "bad data_offsets")


def test_rejects_bad_shapes_and_offset_lists():
    rejects(build({"t": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, bytes(4)),
            "shape must be an array of non-negative integers")
    rejects(build({"t": {"dtype": "F32", "shape": [1.5], "data_offsets": [0, 4]}}, bytes(4)),
            "shape must be an array")
    rejects(build({"t": {"dtype": "F32", "shape": [1], "data_offsets": [0]}}, bytes(4)),
            "data_offsets must be a pair")


def test_rejects_overlapping_tensors():
    rejects(build({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]},
                   "b": {"dtype": "F32", "shape": [4], "data_offsets": [8, 24]}}, bytes(24)), "b overlaps a")


def test_reads_a_tensor_stored_at_a_non_zero_offset():
    data = np.array([9, 9, 1, 2, 3], np.float32).tobytes()
    st = b2a.Safetensors.fromBytes(build({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
                                          "b": {"dtype": "F32", "shape": [3], "data_offsets": [8, 20]}}, data))
    assert st.readF32("b").tolist() == [1, 2, 3]
    assert st.names() == ["a", "b"]


def test_widens_bf16_f16_and_f64():
    # bf16: 0x3f80 is 1.0, 0xc000 is -2.0, 0x0000 is +0 (test/safetensors.test.js:110-118)
    st = b2a.Safetensors.fromBytes(build({"t": {"dtype": "BF16", "shape": [3], "data_offsets": [0, 6]}},
                                         np.array([0x3f80, 0xc000, 0x0000], np.uint16).tobytes()))
    assert st.readF32("t").tolist() == [1, -2, 0]
    h = np.array([1.5, -0.0, 65504, 6e-8, np.inf], np.float16)
    st = b2a.Safetensors.fromBytes(b2a.write_safetensors({"h": h}))
    assert np.array_equal(st.readF32("h"), h.astype(np.float32))
    d = np.array([0.1, 1e-40, 3.4e38, -2.5], np.float64)
    st = b2a.Safetensors.fromBytes(b2a.write_safetensors({"d": d}))
    assert np.array_equal(st.readF32("d"), d.astype(np.float32))
    st = b2a.Safetensors.fromBytes(b2a.write_safetensors({"i": np.arange(4, dtype=np.int8)}))
    with pytest.raises(b2a.B2AError, match="cannot widen I8 to f32"):
        st.readF32("i")
    assert st.readRaw("i") == bytes([0, 1, 2, 3])


def test_names_a_missing_tensor_in_the_error():
    st = b2a.Safetensors.fromBytes(build(OK, bytes(16)))
    with pytest.raises(b2a.B2AError, match='no tensor named "nope"'):
        st.info("nope")


def test_opens_a_file_from_disk(tmp_path):
    data = np.arange(12, dtype=np.float32).reshape(3, 4)
    path = tmp_path / "m.safetensors"
    path.write_bytes(b2a.write_safetensors({"x": data, "y": np.ones(2, np.float32)}))
    st = b2a.Safetensors.open(str(path))
    assert st.names() == ["x", "y"]
    assert np.array_equal(st.readF32("x"), data)
    st.close()
    with pytest.raises(b2a.B2AError, match="cannot open"):
        b2a.Safetensors.open(str(tmp_path / "missing.safetensors"))


def test_qwen25_inventory_matches_the_real_checkpoint():
    golden = json.load(open(os.path.join(HERE, "golden", "qwen25_tensors.json")))
    want = b2a.ModelConfig.qwen25_05b(max_position_embeddings=32768).expectedTensors()
    assert len(want) == golden["tensor_count"] == 290
    assert sorted(want) == sorted(golden["tensors"])
    for name, t in golden["tensors"].items():
        assert tuple(t["shape"]) == want[name], name
        assert t["dtype"] == "BF16"
    # every byte of the file is a header or a tensor: a ~30 KB header remains
    data = sum(2 * int(np.prod(t["shape"])) for t in golden["tensors"].values())
    header = golden["file_bytes"] - 8 - data
    assert 10_000 < header < 100_000
    assert b2a.ModelConfig.qwen25_05b().parameterCount() == data // 2
