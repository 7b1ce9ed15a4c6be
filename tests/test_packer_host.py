"""Host side of the direct AutoRound load (no GPU): the AR4 header that
export_autoround_for_cpp.py writes is unpacked as the reference packer does
(scripts/autoround_pack_llama2_u250.py main(), :382-386, which asserts the
magic), and streams with a wrong magic, a geometry other than the
Llama-2-7B shape the library is built for, or a short read are refused
before any device work."""
import importlib
import io
import struct

import pytest

packer = importlib.import_module("4pe_u250_b200.packer")


def _header(magic=b"AR4\0", ver=1, dim=4096, hidden=11008, layers=32, heads=32, kv=32, vocab=32000, group=128):
    h = struct.pack("<4sIIIIIIII", magic, ver, dim, hidden, layers, heads, kv, vocab, group)
    return h + b"\0" * (packer.HEADER_BYTES - len(h))


def test_header_fields():
    hdr = packer.read_header(io.BytesIO(_header(layers=2)))
    assert hdr == {"version": 1, "dim": 4096, "hidden": 11008, "layers": 2, "heads": 32, "kv_heads": 32,
                   "vocab": 32000, "group": 128}


@pytest.mark.parametrize("kw", [{"magic": b"AR5\0"}, {"dim": 2048}, {"hidden": 11264}, {"vocab": 32256},
                                {"group": 32}, {"layers": 0}, {"layers": 33}])
def test_header_rejects(kw):
    with pytest.raises(ValueError):
        packer.read_header(io.BytesIO(_header(**kw)))


def test_truncated_streams():
    with pytest.raises(ValueError):
        packer.read_header(io.BytesIO(_header()[:100]))
    f = io.BytesIO(b"\0" * 10)
    with pytest.raises(ValueError):
        packer._read(f, "<f4", 4)
