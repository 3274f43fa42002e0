"""Safetensors index on the host (no GPU): mrt_safetensors_open / count /
name / info / read-to-host against files written here, and the error cases of
the reference's SafeTensorsFile (src/loader/safetensors.cpp:23-28, 33-69,
71-131) plus the bounds checks it leaves out."""
import json
import os
import struct

import numpy as np
import pytest

from mruntime_b200 import capi


def _write(path, header: dict, data: bytes, pad_header: bool = True) -> None:
    hb = json.dumps(header).encode()
    if pad_header:
        hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        f.write(data)


def _ok_file(tmp_path):
    a = np.arange(12, dtype=np.float16).reshape(3, 4)
    b = (np.arange(5, dtype=np.uint16) + 0x3F80).astype(np.uint16)  # BF16 bit patterns
    c = np.linspace(-1, 1, 6, dtype=np.float32).reshape(2, 3)
    data = a.tobytes() + b.tobytes() + c.tobytes()
    o1 = a.nbytes
    o2 = o1 + b.nbytes
    hdr = {"__metadata__": {"format": "pt", "nested": {"k": [1, 2.5e-3, True, None, "é\\\"x"]}},
           "model.a": {"dtype": "F16", "shape": [3, 4], "data_offsets": [0, o1]},
           "b.bias": {"dtype": "BF16", "shape": [5], "data_offsets": [o1, o2]},
           "cé": {"dtype": "F32", "shape": [2, 3], "data_offsets": [o2, o2 + c.nbytes]}}
    p = str(tmp_path / "ok.safetensors")
    _write(p, hdr, data)
    return p, a, b, c


def test_index_and_host_read(tmp_path):
    p, a, b, c = _ok_file(tmp_path)
    f = capi.SafeTensors(p)
    assert f.names() == sorted(["model.a", "b.bias", "cé"])  # the reference's std::map order
    assert f.info("model.a") == (capi.FP16, (3, 4), a.nbytes)
    assert f.info("b.bias") == (capi.BF16, (5,), b.nbytes)
    assert f.info("cé") == (capi.FP32, (2, 3), c.nbytes)
    out = np.zeros(6, np.float32)
    f.read("cé", out.ctypes.data, out.nbytes)
    np.testing.assert_array_equal(out, c.reshape(-1))
    with pytest.raises(capi.MrtError) as e:
        f.read("cé", out.ctypes.data, out.nbytes - 4)
    assert e.value.code == 2
    with pytest.raises(capi.MrtError) as e:
        f.info("missing")
    assert e.value.code == 1 and "no tensor" in str(e.value)
    f.close()


@pytest.mark.parametrize("case,code,text", [
    ("dtype", 1, "Unsupported dtype: I64"),
    ("offsets3", 1, "exactly 2"),
    ("past_eof", 1, "past the end"),
    ("size", 1, "does not match"),
    ("not_object", 1, "must be an object"),
    ("bad_json", 1, "Failed to parse SafeTensors header JSON"),
    ("header_len", 1, "Invalid header size"),
    ("tiny", 1, "File too small"),
    ("missing", 1, "Failed to open file"),
])
def test_open_errors(tmp_path, case, code, text):
    p = str(tmp_path / f"{case}.safetensors")
    data = np.zeros(8, np.uint16).tobytes()
    if case == "dtype":
        _write(p, {"t": {"dtype": "I64", "shape": [2], "data_offsets": [0, 16]}}, data)
    elif case == "offsets3":
        _write(p, {"t": {"dtype": "F16", "shape": [8], "data_offsets": [0, 8, 16]}}, data)
    elif case == "past_eof":
        _write(p, {"t": {"dtype": "F16", "shape": [16], "data_offsets": [0, 32]}}, data)
    elif case == "size":
        _write(p, {"t": {"dtype": "F16", "shape": [3], "data_offsets": [0, 16]}}, data)
    elif case == "not_object":
        _write(p, [1, 2], data)
    elif case == "bad_json":
        with open(p, "wb") as f:
            f.write(struct.pack("<Q", 9) + b'{"t": [1,' + data)
    elif case == "header_len":
        with open(p, "wb") as f:
            f.write(struct.pack("<Q", 1 << 40) + b"{}")
    elif case == "tiny":
        with open(p, "wb") as f:
            f.write(b"abc")
    with pytest.raises(capi.MrtError) as e:
        capi.SafeTensors(p)
    assert e.value.code == code and text in str(e.value), str(e.value)
    if case in ("dtype", "offsets3", "past_eof", "size"):
        assert "'t'" in str(e.value)  # the failing tensor is named, as in the reference's message


def test_checkpoint_written_for_the_goldens_indexes(tmp_path):
    """The seeded decoder checkpoint writer (tests/golden/gen_decode_7b.py)
    produces files this loader indexes with every tensor's shape."""
    import sys

    from conftest import GOLDEN
    from mruntime_b200 import workloads as W

    sys.path.insert(0, GOLDEN)
    import gen_decode_7b as G

    paths = G.write_checkpoint(str(tmp_path), W.DECODER_TINY, 3, 16)
    f = capi.SafeTensors(paths["model"])
    specs = {n: s for n, s, _ in W.decoder_tensor_specs(W.DECODER_TINY)}
    assert set(f.names()) == set(specs)
    for name, shape in specs.items():
        assert f.info(name)[:2] == (capi.FP16, tuple(shape))
    f.close()
