"""Snapshot reader (coli_cuda_st_*) on the host: index, shapes, dtype
conversion and rejection of malformed files. No device needed."""
import json
import os
import struct

import numpy as np
import pytest

from conftest import load_pkg
import st_writer


@pytest.fixture(scope="module")
def lib():
    return load_pkg().load_library()


def _snap(tmp_path, tensors, files=1):
    names = list(tensors)
    for k in range(files):
        part = {n: tensors[n] for n in names[k::files]}
        st_writer.write(str(tmp_path / f"model-{k:05d}.safetensors"), part, metadata={"format": "pt"})
    (tmp_path / "config.json").write_text(json.dumps({"num_hidden_layers": 1}))
    return str(tmp_path)


def test_index_and_conversion(lib, tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((96, 40)).astype(np.float32)
    b = rng.standard_normal(257).astype(np.float32)
    c = rng.standard_normal((3, 5, 7)).astype(np.float32)
    snap = load_pkg().snapshot.Snapshot(lib, _snap(tmp_path, {"w.bf16": ("BF16", a), "v.f16": ("F16", b),
                                                              "t.f32": ("F32", c), "q.i8": ("I8", np.ones(4))},
                                                   files=2))
    assert snap.info("w.bf16") == ((96, 40), 0)
    assert snap.info("v.f16") == ((257,), 1)
    assert snap.info("t.f32") == ((3, 5, 7), 2)
    assert snap.info("missing") is None
    np.testing.assert_array_equal(snap.read("w.bf16"), st_writer.bf16_value(a))
    np.testing.assert_array_equal(snap.read("v.f16"), b.astype(np.float16).astype(np.float32))
    np.testing.assert_array_equal(snap.read("t.f32"), c)
    out = np.zeros(10, np.float32)
    assert lib.coli_cuda_st_read_f32(snap.h, b"t.f32", out.ctypes.data_as(load_pkg().coli_cuda._fp), 10) == -1
    assert b"105 elements" in lib.coli_cuda_last_error()
    assert lib.coli_cuda_st_read_f32(snap.h, b"q.i8", out.ctypes.data_as(load_pkg().coli_cuda._fp), 10) == -1
    snap.close()


def test_subnormal_and_special_halves(lib, tmp_path):
    h = np.array([0.0, -0.0, 6e-8, 3e-5, 65504.0, np.inf, -np.inf, 1.0, -2.5], np.float16)
    snap = load_pkg().snapshot.Snapshot(lib, _snap(tmp_path, {"h": ("F16", h)}))
    np.testing.assert_array_equal(snap.read("h"), h.astype(np.float32))
    snap.close()


@pytest.mark.parametrize("corrupt", ["offsets_beyond_file", "shape_vs_bytes", "header_length", "not_json"])
def test_malformed_files_are_refused(lib, tmp_path, corrupt):
    path = tmp_path / "bad.safetensors"
    data = np.zeros(16, np.float32).tobytes()
    hdr = {"x": {"dtype": "F32", "shape": [16], "data_offsets": [0, 64]}}
    if corrupt == "offsets_beyond_file":
        hdr["x"]["data_offsets"] = [0, 4096]
    if corrupt == "shape_vs_bytes":
        hdr["x"]["shape"] = [17]
    h = json.dumps(hdr).encode() if corrupt != "not_json" else b"[1, 2, 3]"
    n = len(h) if corrupt != "header_length" else 1 << 40
    path.write_bytes(struct.pack("<Q", n) + h + data)
    assert lib.coli_cuda_st_open(str(tmp_path).encode()) == -1
    assert lib.coli_cuda_last_error()


def test_missing_directory(lib):
    assert lib.coli_cuda_st_open(b"/nonexistent/snapshot") == -1
