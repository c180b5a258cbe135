"""Property tests of the C++ safetensors header parser (include/nvfp4_loader.h)
on generated headers: every valid header (arbitrary tensor names with quotes,
backslashes, braces and non-ASCII characters, either JSON escaping, any
whitespace, metadata strings with brackets) parses to exactly its tensors,
and every corruption of one is either parsed or refused with an error,
never a crash.  Host-side only: no GPU."""
import json
import os
import struct
import tempfile

import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

DTYPES = {"U8": 1, "I8": 1, "BOOL": 1, "F8_E4M3": 1, "BF16": 2, "F16": 2, "I16": 2, "F32": 4,
          "I32": 4, "F64": 8, "I64": 8}

names = st.text(alphabet=st.characters(blacklist_categories=("Cs",), min_codepoint=32,
                                       max_codepoint=0x2FFF) | st.sampled_from('"\\{}[],:'),
                min_size=1, max_size=24).filter(lambda s: s != "__metadata__")
tensor = st.tuples(st.sampled_from(sorted(DTYPES)),
                   st.lists(st.integers(0, 5), min_size=0, max_size=3))
checkpoint = st.tuples(st.dictionaries(names, tensor, min_size=1, max_size=6),
                       st.dictionaries(st.text(max_size=8), st.text(max_size=16), max_size=3),
                       st.booleans(), st.sampled_from([None, 0, 1, 2]))


def build(tensors, metadata, ascii_only, indent):
    header, offset = {}, 0
    if metadata:
        header["__metadata__"] = metadata
    for name, (dt, shape) in tensors.items():
        n = DTYPES[dt]
        for d in shape:
            n *= d
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [offset, offset + n]}
        offset += n
    text = json.dumps(header, ensure_ascii=ascii_only, indent=indent)
    return text.encode(), bytes(i % 251 for i in range(offset)), header


def write(path, hb, data, size=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb) if size is None else size))
        f.write(hb)
        f.write(data)


@settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(checkpoint)
def test_valid_headers_parse_exactly(ck):
    from nvfp4 import weight_loader as W

    tensors, metadata, ascii_only, indent = ck
    hb, data, header = build(tensors, metadata, ascii_only, indent)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.safetensors")
        write(p, hb, data)
        f = W.open_safetensors(p)
        try:
            got = {t.name: (t.dtype, list(t.shape), t.data_offset, t.data_size) for t in f.tensors}
            want = {k: (v["dtype"], v["shape"], v["data_offsets"][0],
                        v["data_offsets"][1] - v["data_offsets"][0])
                    for k, v in header.items() if k != "__metadata__"}
            assert got == want
            assert [t.name for t in f.tensors] == [k for k in header if k != "__metadata__"]
            for i, t in enumerate(f.tensors):
                assert f.find_tensor(t.name) == i
        finally:
            f.close()


@settings(max_examples=200, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(checkpoint, st.integers(0, 10 ** 6), st.integers(0, 255),
       st.sampled_from(["truncate", "flip", "insert", "size"]))
def test_corrupt_headers_never_crash(ck, where, byte, how):
    from nvfp4 import _lib
    from nvfp4 import weight_loader as W

    tensors, metadata, ascii_only, indent = ck
    hb, data, _ = build(tensors, metadata, ascii_only, indent)
    pos = where % (len(hb) + 1)
    size = None
    if how == "truncate":
        hb = hb[:pos]
    elif how == "flip" and hb:
        i = min(pos, len(hb) - 1)
        hb = hb[:i] + bytes([byte]) + hb[i + 1:]
    elif how == "insert":
        hb = hb[:pos] + bytes([byte]) + hb[pos:]
    else:
        size = where  # a length field that disagrees with the header
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.safetensors")
        write(p, hb, data, size)
        try:
            f = W.open_safetensors(p)
        except _lib.Nvfp4Error:
            return
        for t in f.tensors:
            assert t.data_size >= 0 and t.data_offset >= 0
        f.close()


@pytest.mark.parametrize("raw,ok", [
    (b'{"a\xff":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', False),      # invalid UTF-8
    (b'{"a\xc0\x80":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', False),  # overlong NUL
    (b'{"a\xed\xa0\x80":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', False),  # surrogate
    (b'{"a\\udc00":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', False),   # lone low surrogate
    (b'{"a\\u0000b":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', False),  # NUL in a name
    (b'{"a":{"dtype":"U\\u00008","shape":[1],"data_offsets":[0,1]}}', False),   # NUL in a dtype
    (b'{"__metadata__":{"k":"\\u0000"},"a":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}',
     True),                                                                       # NUL in metadata
    (b'{"\xc3\xa9\xf0\x9f\x98\x80":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', True),
])
def test_header_text_rules(raw, ok):
    """The header must be well-formed UTF-8 JSON; tensor names and dtypes
    cannot hold NUL (they cross the C ABI as C strings).  Metadata values
    are skipped, whatever they hold."""
    from nvfp4 import _lib
    from nvfp4 import weight_loader as W

    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.safetensors")
        write(p, raw, b"\x07")
        if ok:
            f = W.open_safetensors(p)
            assert len(f.tensors) == 1 and f.tensors[0].data_size == 1
            f.close()
        else:
            with pytest.raises(_lib.Nvfp4Error):
                W.open_safetensors(p)
