"""Safetensors checkpoints through the C ABI (gm_checkpoint_*), on CPU: files
in the reference writer's layout and in the standard safetensors writer's,
sharded directories, and every malformed-header case the reader must refuse
(safetensors/parser.mojo: header length bound, offsets inside the data, byte
counts equal to shape x dtype size)."""
import json
import os

import numpy as np
import pytest

import gmoe
from helpers import write_safetensors


def _sample(rng):
    return [
        ("model.language_model.layers.0.experts.gate_up_proj",
         rng.integers(-127, 128, size=(96, 64), dtype=np.int8), None, None),
        ("model.language_model.layers.0.experts.gate_up_proj.scale",
         rng.random(96, dtype=np.float32), None, None),
        ("model.language_model.layers.0.router.scale",
         rng.integers(0, 1 << 16, size=(40,), dtype=np.uint16), None, [40, 1]),
        ("cube", rng.integers(0, 1 << 16, size=(3, 5, 8), dtype=np.uint16), "BF16", None),
        ("scalar", np.array([0x3F80], np.uint16), "BF16", []),
        ("empty", np.zeros((0, 16), np.float32), None, None),
        ("ids", rng.integers(-5, 5, size=(7,), dtype=np.int64), None, None),
    ]


def _fold(a):
    if a.ndim == 0:
        return a.reshape(1, 1)
    if a.ndim == 1:
        return a.reshape(-1, 1)
    return a.reshape(-1, a.shape[-1])


def _check_all(ck, entries):
    assert ck.names() == sorted(n for n, *_ in entries)
    for name, arr, tag, shape in entries:
        arr = np.asarray(arr)
        want_tag = tag or ("BF16" if arr.dtype == np.uint16 else None)
        got_tag, got_shape = ck.info(name)
        if want_tag:
            assert got_tag == want_tag
        assert got_shape == tuple(arr.shape if shape is None else shape)
        f = _fold(arr.reshape(shape) if shape is not None else arr)
        out = np.empty_like(f)
        ck.read_rows(name, 0, f.shape[0], out)
        assert np.array_equal(out, f)
        if f.shape[0] >= 3:  # a middle row block
            part = np.empty_like(f[1:3])
            ck.read_rows(name, 1, 2, part)
            assert np.array_equal(part, f[1:3])


def test_reference_layout_file(tmp_path):
    entries = _sample(np.random.default_rng(1))
    p = write_safetensors(tmp_path / "model.safetensors", entries)
    with gmoe.Checkpoint(p) as ck:
        _check_all(ck, entries)


def test_reference_layout_is_standard_safetensors(tmp_path):
    """The restated writer's file reads back with the safetensors package."""
    safetensors_numpy = pytest.importorskip("safetensors.numpy")
    entries = [e for e in _sample(np.random.default_rng(2)) if e[2] != "BF16"
               and not e[0].endswith("router.scale")]
    p = write_safetensors(tmp_path / "m.safetensors", entries)
    back = safetensors_numpy.load_file(str(p))
    for name, arr, _, _ in entries:
        assert np.array_equal(back[name], arr)


def test_standard_writer_with_metadata(tmp_path):
    """Files of the standard writer (metadata, alignment padding, bf16 from
    torch) read through the C reader."""
    torch = pytest.importorskip("torch")
    st_torch = pytest.importorskip("safetensors.torch")
    g = torch.Generator().manual_seed(3)
    tensors = {
        "a.weight": torch.randn(33, 17, generator=g).to(torch.bfloat16),
        "b.scale": torch.rand(9, generator=g),
        "c.q": torch.randint(-128, 127, (4, 6, 10), generator=g, dtype=torch.int8),
    }
    p = tmp_path / "std.safetensors"
    st_torch.save_file(tensors, str(p), metadata={"format": "pt", "note": "x\"y\\u00e9"})
    with gmoe.Checkpoint(p) as ck:
        assert ck.names() == sorted(tensors)
        assert ck.info("a.weight") == ("BF16", (33, 17))
        assert ck.info("c.q") == ("I8", (4, 6, 10))
        out = np.empty((33, 17), np.uint16)
        ck.read_rows("a.weight", 0, 33, out)
        assert np.array_equal(out, tensors["a.weight"].view(torch.int16).numpy().view(np.uint16))
        q = np.empty((24, 10), np.int8)
        ck.read_rows("c.q", 0, 24, q)
        assert np.array_equal(q, tensors["c.q"].numpy().reshape(24, 10))


def test_sharded_directory(tmp_path):
    rng = np.random.default_rng(4)
    e = _sample(rng)
    d = tmp_path / "ckpt"
    d.mkdir()
    write_safetensors(d / "model-00001-of-00002.safetensors", e[:3])
    write_safetensors(d / "model-00002-of-00002.safetensors", e[3:])
    (d / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {n: "x" for n, *_ in e}}))
    with gmoe.Checkpoint(d) as ck:
        _check_all(ck, e)
    # a tensor in two shards is refused
    write_safetensors(d / "model-00003-of-00003.safetensors", e[:1])
    with pytest.raises(gmoe.GmoeError, match="appears twice"):
        gmoe.Checkpoint(d)


def test_empty_directory_refused(tmp_path):
    with pytest.raises(gmoe.GmoeError, match="no .safetensors"):
        gmoe.Checkpoint(tmp_path)
    with pytest.raises(gmoe.GmoeError):
        gmoe.Checkpoint(tmp_path / "missing.safetensors")


def _raw_file(path, header_bytes, data=b"", length=None):
    n = len(header_bytes) if length is None else length
    path.write_bytes(n.to_bytes(8, "little") + header_bytes + data)
    return path


@pytest.mark.parametrize("header,data,length,match", [
    (b'{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,16]}}', b"\0" * 8, None, "outside"),
    (b'{"t":{"dtype":"F32","shape":[3],"data_offsets":[0,16]}}', b"\0" * 16, None, "differs"),
    (b'{"t":{"dtype":"Q7","shape":[4],"data_offsets":[0,4]}}', b"\0" * 4, None, "unknown dtype"),
    (b'{"t":{"dtype":"F32","shape":[-1],"data_offsets":[0,4]}}', b"\0" * 4, None, "negative"),
    (b'{"t":{"dtype":"F32","shape":[1.5],"data_offsets":[0,4]}}', b"\0" * 4, None, "fraction"),
    (b'{"t":{"dtype":"F32","shape":[1]}}', b"\0" * 4, None, "lacks"),
    (b'{"t":{"dtype":"F32","shape":[1],"data_offsets":[4,0]}}', b"\0" * 4, None, "outside"),
    (b'{"t":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}', b"\0" * 4, None, "expected"),
    (b'{"t":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}} x', b"\0" * 4, None, "trailing"),
    (b'{"t\x01":{}}', b"", None, "control"),
    (b'{}', b"", 1 << 40, "exceeds"),
    (b'{}', b"", 200 << 20, "exceeds"),
    (b'{}', b"", 64, "exceeds the file"),
])
def test_malformed_headers_refused(tmp_path, header, data, length, match):
    p = _raw_file(tmp_path / "bad.safetensors", header, data, length)
    with pytest.raises(gmoe.GmoeError, match=match):
        gmoe.Checkpoint(p)


def test_short_file_refused(tmp_path):
    p = tmp_path / "short.safetensors"
    p.write_bytes(b"\x02\0\0")
    with pytest.raises(gmoe.GmoeError, match="shorter"):
        gmoe.Checkpoint(p)


def test_metadata_and_escapes(tmp_path):
    hdr = (b'{"__metadata__":{"format":"pt","k":"\\"\\\\\\/\\b\\f\\n\\r\\t\\u00e9\\ud83d\\ude00"},'
           b'"na\\u00efve":{"dtype":"U8","shape":[2,2],"data_offsets":[0,4]}}')
    p = _raw_file(tmp_path / "m.safetensors", hdr, b"\x01\x02\x03\x04")
    with gmoe.Checkpoint(p) as ck:
        assert ck.names() == ["naïve"]
        out = np.empty((2, 2), np.uint8)
        ck.read_rows("naïve", 0, 2, out)
        assert out.tolist() == [[1, 2], [3, 4]]


def test_read_errors(tmp_path):
    e = _sample(np.random.default_rng(5))
    p = write_safetensors(tmp_path / "m.safetensors", e)
    with gmoe.Checkpoint(p) as ck:
        name = e[0][0]
        with pytest.raises(gmoe.GmoeError, match="outside"):
            ck.read_rows(name, 90, 7, np.empty((7, 64), np.int8))
        with pytest.raises(gmoe.GmoeError, match="outside"):
            ck.read_rows(name, -1, 1, np.empty((1, 64), np.int8))
        with pytest.raises(gmoe.GmoeError, match="needed"):
            ck.read_rows(name, 0, 2, np.empty((1, 64), np.int8))
        with pytest.raises(gmoe.GmoeError, match="not in the checkpoint"):
            ck.info("nope")
        ck.read_rows(name, 96, 0, np.empty((0, 64), np.int8))  # empty read at the end


def test_large_tensor_threaded_read(tmp_path):
    """Reads above the threading threshold (8 MiB pieces) return every byte."""
    rng = np.random.default_rng(6)
    big = rng.integers(-128, 128, size=(1409, 2816 * 9), dtype=np.int8)  # ~36 MB
    p = write_safetensors(tmp_path / "big.safetensors", [("pad", np.zeros(3, np.uint8), None, None),
                                                          ("big", big, None, None)])
    with gmoe.Checkpoint(p) as ck:
        out = np.empty_like(big)
        ck.read_rows("big", 0, big.shape[0], out)
        assert np.array_equal(out, big)
        part = np.empty((700, big.shape[1]), np.int8)
        ck.read_rows("big", 333, 700, part)
        assert np.array_equal(part, big[333:1033])
    os.remove(p)


def test_utf8_names(tmp_path):
    """Header strings are UTF-8 (the safetensors format): raw multi-byte
    sequences are kept as they are, malformed ones (a stray continuation
    byte, an overlong form, an encoded surrogate, a truncated sequence)
    refuse the file."""
    name = "exp\u00e9rt.\U0001F600"
    hdr = ('{"%s":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}' % name).encode()
    with gmoe.Checkpoint(_raw_file(tmp_path / "ok.safetensors", hdr, b"\x07")) as ck:
        assert ck.names() == [name]
        out = np.empty((1, 1), np.uint8)
        ck.read_rows(name, 0, 1, out)
        assert out[0, 0] == 7
    for bad in (b"\xff", b"\x80", b"\xc0\xaf", b"\xed\xa0\x80", b"\xf4\x90\x80\x80", b"\xe2\x82"):
        hdr = b'{"a' + bad + b'":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}'
        with pytest.raises(gmoe.GmoeError, match="UTF-8"):
            gmoe.Checkpoint(_raw_file(tmp_path / "bad.safetensors", hdr, b"\x07"))


def test_mutated_headers_never_crash(tmp_path):
    """Seeded mutations of a valid header (byte swaps, insertions, deletions,
    deep nesting, short data, wrong header lengths): every open either
    succeeds with readable tensors or fails with an error status."""
    import random
    good = (b'{"__metadata__":{"format":"pt"},"a":{"dtype":"BF16","shape":[2,3],"data_offsets":[0,12]},'
            b'"b":{"dtype":"F32","shape":[4],"data_offsets":[12,28]}}')
    data = bytes(range(28))
    rng = random.Random(1234)
    alphabet = b'{}[]":,0123456789-+.eE \\u\x00\x01\x80\xc3\xa9\xffabcdefghFBIU'
    p = tmp_path / "f.safetensors"
    opened = refused = 0
    for _ in range(3000):
        h = bytearray(good)
        for _ in range(rng.randint(1, 6)):
            op, i = rng.random(), rng.randrange(len(h) + 1)
            if op < 0.4 and h:
                h[min(i, len(h) - 1)] = rng.choice(alphabet)
            elif op < 0.6:
                h[i:i] = bytes(rng.choice(alphabet) for _ in range(rng.randint(1, 8)))
            elif op < 0.8:
                del h[i:i + rng.randint(1, 8)]
            else:
                h[i:i] = b"[" * rng.randint(1, 200)
        d = data[:rng.randint(0, len(data))] if rng.random() < 0.2 else data
        n = len(h) if rng.random() < 0.9 else rng.randint(0, 1 << 20)
        p.write_bytes(n.to_bytes(8, "little") + bytes(h) + d)
        try:
            with gmoe.Checkpoint(p) as ck:
                for nm in ck.names():
                    _, shape = ck.info(nm)
                    rows = shape[0] if shape else 1
                    buf = np.zeros(max(int(np.prod(shape)) * 8, 64), np.uint8)
                    try:
                        ck.read_rows(nm, 0, rows, buf)
                    except gmoe.GmoeError:
                        pass
            opened += 1
        except gmoe.GmoeError:
            refused += 1
    assert opened > 10 and refused > 1000
