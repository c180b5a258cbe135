"""The C++ safetensors reader (include/nvfp4_loader.h) against the restated
reference loader (oracle/safetensors_ref.py, nvfp4/weight_loader.mojo) and
the `safetensors` package's own reader, on files the package writes and on
hand-written headers.  Host-side only: no GPU."""
import ctypes
import os
import struct

import numpy as np
import pytest
import torch

import st_fixtures as F


@pytest.fixture(scope="module")
def R():
    from oracle import safetensors_ref

    return safetensors_ref


@pytest.fixture(scope="module")
def W():
    from nvfp4 import weight_loader

    return weight_loader


def mixed_checkpoint(path):
    rng = np.random.default_rng(0)
    t = {}
    w, sf = F.rand_linear(rng, 64, 256)
    F.nvfp4_linear(t, "model.layers.0.mlp.experts.0.gate_proj", w, sf, ws2=np.float32(3e-3),
                   ins=np.float32(0.5))
    w2, sf2 = F.rand_linear(rng, 32, 128)
    F.nvfp4_linear(t, "model.layers.0.self_attn.q_proj", w2, sf2,
                   ws2=rng.uniform(1e-3, 1e-2, 32).astype(np.float32))
    t["model.layers.0.mlp.gate.weight"] = torch.randn(8, 256).to(torch.bfloat16)
    t["model.norm.weight"] = torch.randn(256).to(torch.bfloat16)
    t["scalar_i64"] = torch.tensor(7, dtype=torch.int64)
    t["empty"] = torch.zeros((0, 4), dtype=torch.float32)
    F.save(path, t, metadata={"format": "pt", "note": "plain text"})
    return t


def test_header_matches_reference_and_safetensors(tmp_path, R, W):
    from safetensors import safe_open

    p = tmp_path / "model.safetensors"
    t = mixed_checkpoint(p)
    ours = W.open_safetensors(str(p))
    ref = R.open_safetensors(str(p))
    assert [x.name for x in ours.tensors] == [x.name for x in ref.tensors]
    for a, b in zip(ours.tensors, ref.tensors):
        assert (a.dtype, a.shape, a.data_offset, a.data_size) == \
            (b.dtype, b.shape, b.data_offset, b.data_size), a.name
    with safe_open(str(p), "pt") as f:
        assert sorted(f.keys()) == sorted(x.name for x in ours.tensors)
        for x in ours.tensors:
            assert list(f.get_slice(x.name).get_shape()) == x.shape
            assert f.get_slice(x.name).get_dtype() == x.dtype
            raw = f.get_tensor(x.name).contiguous().reshape(-1).view(torch.uint8).numpy().tobytes() \
                if x.data_size else b""
            assert ours.read_tensor_bytes(ours.find_tensor(x.name)).tobytes() == raw
            assert raw == ref.read_tensor_bytes(ref.find_tensor(x.name))
    assert ours.find_tensor("missing") == -1 and not ours.has_tensor("missing")
    ours.close()


def test_metadata_with_braces(tmp_path, R, W):
    """A `}` inside a __metadata__ string: the reference's brace counting does
    not skip strings (nvfp4/weight_loader.mojo:321-335), so it loses every
    tensor after it; the C++ parser reads the JSON properly."""
    p = tmp_path / "model.safetensors"
    F.save(p, {"a": torch.arange(6, dtype=torch.float32)},
           metadata={"note": "braces } { and \"quotes\""})
    assert [x.name for x in W.open_safetensors(str(p)).tensors] == ["a"]
    assert [x.name for x in R.open_safetensors(str(p)).tensors] == []


def test_hand_written_headers(tmp_path, R, W):
    """Whitespace, key order inside a tensor entry, escapes in names; the
    reference's scanning parser and the C++ JSON parser agree."""
    data = bytes(range(48))
    hdr = ('{\n  "__metadata__" : {"a": "b"},\n'
           '  "x.weight" : { "data_offsets" : [ 0 , 16 ] ,\t"shape":[4, 4], "dtype" : "U8" },\n'
           '  "y\\u00e9" : {"dtype":"F32","shape":[ ],"data_offsets":[16,20]},\n'
           '  "z" : {"dtype":"BF16","shape":[2,2,3],"data_offsets":[20,44]}\n}')
    p = tmp_path / "h.safetensors"
    F.raw_file(p, hdr, data)
    ours = W.open_safetensors(str(p))
    ref = R.open_safetensors(str(p))
    assert [x.name for x in ours.tensors] == ["x.weight", "yé", "z"]
    for a, b in zip(ours.tensors, ref.tensors):
        assert (a.dtype, a.shape, a.data_offset, a.data_size) == \
            (b.dtype, b.shape, b.data_offset, b.data_size)
    assert ours.read_tensor_bytes(2).tobytes() == data[20:44]
    ours.close()


@pytest.mark.parametrize("header,size", [
    ('{"a":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}', 0),         # zero header size
    ('{"a":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}', 10 ** 6),   # beyond the file
    ('{"a":{"dtype":"U8","shape":[4],"data_offsets":[0,4]', None),        # truncated JSON
    ('{"a":{"dtype":"U8","shape":[4],"data_offsets":[0,400]}}', None),    # data past the end
    ('{"a":{"dtype":"U8","shape":[4],"data_offsets":[4,0]}}', None),      # end < begin
    ('{"a":{"dtype":"U8","shape":[-4],"data_offsets":[0,4]}}', None),     # negative dim
])
def test_header_errors(tmp_path, W, header, size):
    from nvfp4 import _lib

    p = tmp_path / "bad.safetensors"
    F.raw_file(p, header, b"\0" * 8, header_size=size)
    with pytest.raises(_lib.Nvfp4Error):
        W.open_safetensors(str(p))


def test_reference_rejects_bad_header_sizes(tmp_path, R):
    p = tmp_path / "bad.safetensors"
    F.raw_file(p, '{}', b"", header_size=0)
    with pytest.raises(ValueError):
        R.open_safetensors(str(p))


def f32_cases():
    rng = np.random.default_rng(5)
    pats = list(rng.integers(0, 2 ** 32, size=4000, dtype=np.uint64).astype(np.uint32))
    pats += [0x00000000, 0x80000000, 0x00000001, 0x807FFFFF, 0x00800000, 0x7F7FFFFF,
             0xFF7FFFFF, 0x7F800000, 0xFF800000, 0x7FC00000, 0x3F800000, 0x3B23D70A]
    return [int(p) for p in pats]


def test_f32_from_bytes_matches_reference(R, W):
    """_read_f32_from_bytes: zero / subnormal -> signed zero, inf / NaN -> 1.0,
    fewer than 4 bytes -> 1.0, every normal value exactly."""
    for bits in f32_cases():
        buf = struct.pack("<I", bits)
        ref = R.read_f32_from_bytes(buf)
        got = np.float32(W.read_f32_from_bytes(buf))
        assert got.tobytes() == ref.tobytes(), hex(bits)
        exp = (bits >> 23) & 0xFF
        if 0 < exp < 255:  # normals: the IEEE value
            assert got.tobytes() == np.frombuffer(buf, np.float32)[0].tobytes()
    for short in (b"", b"\x01", b"\x01\x02\x03"):
        assert W.read_f32_from_bytes(short) == 1.0 == R.read_f32_from_bytes(short)
    # Only the first 4 bytes count.
    assert W.read_f32_from_bytes(struct.pack("<ff", 2.5, 9.0)) == 2.5


def make_shards(d, names):
    os.makedirs(d, exist_ok=True)
    for i, n in enumerate(names):
        F.save(os.path.join(d, n), {f"t{i}": torch.tensor([float(i)])})


@pytest.mark.parametrize("files,ours,ref", [
    (["model.safetensors"], [0], [0]),
    (["model-00001-of-00001.safetensors"], [0], [0]),
    (["model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"], [0, 1], [0, 1]),
    # three shards: the reference's probe loop stops after shard 1
    (["model-00001-of-00003.safetensors", "model-00002-of-00003.safetensors",
      "model-00003-of-00003.safetensors"], [0, 1, 2], [0]),
    # model.safetensors wins over shards in both
    (["model.safetensors", "model-00001-of-00002.safetensors"], [0], [0]),
    # a gap: both stop at the first missing shard
    (["model-00001-of-00004.safetensors", "model-00002-of-00004.safetensors",
      "model-00004-of-00004.safetensors"], [0, 1], [0]),
])
def test_shard_discovery(tmp_path, R, W, files, ours, ref):
    d = str(tmp_path / "m")
    make_shards(d, files)
    assert W.discover_safetensor_shards(d) == [os.path.join(d, files[i]) for i in ours]
    assert R.discover_safetensor_shards(d) == [f"{d}/{files[i]}" for i in ref]
    m = W.open_model_shards(d)
    assert len(m) == len(ours)
    for k, i in enumerate(ours):  # tensor t{i} lives in file i
        assert m.find(f"t{i}") == (k, 0)
    m.close()


def test_shard_discovery_errors(tmp_path, R, W):
    from nvfp4 import _lib

    empty = str(tmp_path / "empty")
    os.makedirs(empty)
    with pytest.raises(_lib.Nvfp4Error):
        W.discover_safetensor_shards(empty)
    with pytest.raises(ValueError):
        R.discover_safetensor_shards(empty)
    # Shard 1 missing: the reference starts from shard 2, this loader refuses.
    d = str(tmp_path / "m")
    make_shards(d, ["model-00002-of-00002.safetensors"])
    assert R.discover_safetensor_shards(d) == [f"{d}/model-00002-of-00002.safetensors"]
    with pytest.raises(_lib.Nvfp4Error):
        W.discover_safetensor_shards(d)


@pytest.mark.parametrize("ws2,ins", [(None, None), (np.float32(2e-3), None),
                                     (np.float32(4e-3), np.float32(0.125)),
                                     ("rows", np.float32(3.0)),
                                     (np.float32(np.inf), np.float32(1e-45))])
def test_linear_info_matches_reference(tmp_path, R, W, ws2, ins):
    rng = np.random.default_rng(3)
    t = {}
    w, sf = F.rand_linear(rng, 48, 512)
    rows = rng.uniform(1e-3, 1e-2, 48).astype(np.float32)
    F.nvfp4_linear(t, "blk.lin", w, sf, ws2=rows if isinstance(ws2, str) else ws2, ins=ins)
    F.save(tmp_path / "model.safetensors", t)
    ref = R.load_linear_safetensors(R.open_safetensors(str(tmp_path / "model.safetensors")),
                                    "blk.lin")
    m = W.open_model_shards(str(tmp_path))
    info = W.linear_info(m, "blk.lin")
    assert (info.out_features, info.in_features) == (ref.out_features, ref.in_features) == (48, 512)
    assert np.float32(info.weight_scale_2).tobytes() == ref.weight_scale_2.tobytes()
    assert np.float32(info.input_scale).tobytes() == ref.input_scale.tobytes()
    assert bool(info.weight_scale_2_rows) == isinstance(ws2, str)
    f = m.shards[info.shard]
    assert f.read_tensor_bytes(f.find_tensor("blk.lin.weight")).tobytes() == ref.packed_weights
    assert f.read_tensor_bytes(f.find_tensor("blk.lin.weight_scale")).tobytes() == ref.blockscales
    m.close()


def test_linear_errors(tmp_path, R, W):
    from nvfp4 import _lib

    rng = np.random.default_rng(4)
    w, sf = F.rand_linear(rng, 16, 64)
    cases = {
        "no_scale": {"a.weight": torch.from_numpy(w)},
        "one_dim": {"a.weight": torch.from_numpy(w.reshape(-1)),
                    "a.weight_scale": torch.from_numpy(sf)},
        "bad_scale_size": {"a.weight": torch.from_numpy(w),
                           "a.weight_scale": torch.from_numpy(sf[:, :2].copy())},
    }
    for name, t in cases.items():
        d = tmp_path / name
        d.mkdir()
        F.save(d / "model.safetensors", t)
        with pytest.raises(ValueError):
            R.load_linear_safetensors(R.open_safetensors(str(d / "model.safetensors")), "a")
        m = W.open_model_shards(str(d))
        with pytest.raises(_lib.Nvfp4Error):
            W.linear_info(m, "a")
        with pytest.raises(_lib.Nvfp4Error):
            W.linear_info(m, "nonexistent")
        m.close()
