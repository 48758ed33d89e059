"""Failure paths of the weight load, on the CPU (no device needed).

The reference rejects a malformed GGUF in gguf.cpp's reader (bad magic, unsupported version,
truncated header or tensor table, tensor data past the end of the file: src/gguf.cpp:73-151) and a
tensor the DiT needs that is absent through WeightSet::need (src/net.mm:110-118, a null buffer plus a
log line). tsn_dit_inspect runs the same checks as tsn_dit_load before any device work and returns
TSN_ERR_FORMAT / TSN_ERR_MISSING / TSN_ERR_IO; the GPU variant of these cases (tsn_dit_load itself,
and a device-side wait made to run out) is in test_gpu_failure.py.

Also here: the oracle library's fixture writer produces the same bytes as the GPU library's, so the
CPU arms that use it read the same weights.
"""
import struct

import pytest

import oracle as O
import tsn
from conftest import SEED, TINY, make_geom

ERR_IO, ERR_FORMAT, ERR_MISSING = 3, 4, 5


@pytest.fixture(scope="module")
def good(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("fail") / "good.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**TINY), SEED)
    return p, open(p, "rb").read()


def _write(tmp_path, name, data):
    p = str(tmp_path / name)
    with open(p, "wb") as f:
        f.write(data)
    return p


def _code(path):
    with pytest.raises(tsn.TsnError) as e:
        tsn.inspect(path)
    return e.value.code, str(e.value)


def test_good_file_inspects(good):
    g, wb = tsn.inspect(good[0])
    assert (g.H, g.NH, g.F, g.depth, g.fused_depth, g.latent_dim) == (256, 4, 512, 3, 1, 64)
    assert wb > 0


def test_missing_file_is_io(tmp_path):
    code, _ = _code(str(tmp_path / "absent.gguf"))
    assert code == ERR_IO


def test_bad_magic_is_format(tmp_path, good):
    data = bytearray(good[1])
    data[0:4] = b"GGUX"
    code, msg = _code(_write(tmp_path, "magic.gguf", data))
    assert code == ERR_FORMAT and "magic" in msg


def test_unsupported_version_is_format(tmp_path, good):
    data = bytearray(good[1])
    data[4:8] = struct.pack("<I", 7)
    code, msg = _code(_write(tmp_path, "ver.gguf", data))
    assert code == ERR_FORMAT and "version" in msg


@pytest.mark.parametrize("where", ["header", "metadata", "tensor_table", "data"])
def test_truncated_file_is_format(tmp_path, good, where):
    from gguf_read import read_header
    data = good[1]
    data_start = read_header(good[0])[3]     # the data section; the tensor table ends < 32 B before it
    cut = {"header": 12, "metadata": 40, "tensor_table": data_start - 40, "data": len(data) - 1000}[where]
    code, msg = _code(_write(tmp_path, f"trunc_{where}.gguf", data[:cut]))
    assert code == ERR_FORMAT, (where, msg)


def test_empty_file_is_io_or_format(tmp_path):
    code, _ = _code(_write(tmp_path, "empty.gguf", b""))
    assert code in (ERR_IO, ERR_FORMAT)


def _renamed(data, name, new):
    """The file with one tensor's name changed in place (same length): that tensor is then absent."""
    assert len(name) == len(new)
    key = struct.pack("<Q", len(name)) + name.encode()
    i = data.rfind(key)          # the tensor table follows the metadata
    assert i > 0
    return data[:i + 8] + new.encode() + data[i + 8 + len(name):]


@pytest.mark.parametrize("name", ["final_layer.conv.weight", "joint_blocks.0.clip_block.attn.qkv.weight",
                                  "fused_blocks.0.ffn.w2.weight", "t_embed.mlp.2.bias"])
def test_missing_tensor_is_missing(tmp_path, good, name):
    new = name[:-1] + ("X" if name[-1] != "X" else "Y")
    code, msg = _code(_write(tmp_path, "missing.gguf", _renamed(good[1], name, new)))
    assert code == ERR_MISSING and name in msg, msg


def test_misshaped_tensor_is_missing(tmp_path, good):
    """A tensor present with the wrong shape (ne[0] of final_layer.conv.weight, [7, H, 64] -> [5, ...])."""
    data = good[1]
    name = "final_layer.conv.weight"
    key = struct.pack("<Q", len(name)) + name.encode()
    i = data.rfind(key) + len(key)
    n_dims = struct.unpack_from("<I", data, i)[0]
    assert n_dims == 3 and struct.unpack_from("<Q", data, i + 4)[0] == 7
    bad = data[:i + 4] + struct.pack("<Q", 5) + data[i + 12:]
    code, msg = _code(_write(tmp_path, "shape.gguf", bad))
    assert code in (ERR_MISSING, ERR_FORMAT) and name in msg, msg


def test_oracle_fixture_writer_matches_library(tmp_path, good):
    p = str(tmp_path / "oracle.gguf")
    O.write_synthetic_gguf(p, seed=SEED, **TINY)
    assert open(p, "rb").read() == good[1]
