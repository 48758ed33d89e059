"""The C-ABI library on the CPU: it loads, exports every symbol include/tsn.h declares, fails
loudly without a GPU, and its GGUF writer/reader handle good and broken files. No compute calls."""
import os
import re

import numpy as np
import pytest

import tsn
from conftest import SEED, TINY, make_geom

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "tsn.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tsn_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = tsn.lib()
    names = declared_symbols()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(names) == set(tsn.EXPORTED), set(names) ^ set(tsn.EXPORTED)


def test_version_and_error_string():
    assert tsn.lib().tsn_version() >= 1
    assert isinstance(tsn.lib().tsn_last_error(), bytes)


def test_no_gpu_fails_loudly():
    """No CPU fallback: without a device the compute entry points return an error."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(tsn.TsnError) as e:
        tsn.Device(0)
    assert e.value.code == 2


def test_synthetic_gguf_roundtrip(tmp_path):
    from gguf_read import read_header
    p = str(tmp_path / "t.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**TINY), SEED)
    _, kv, tensors, data = read_header(p)
    assert kv["dit.hidden_dim"] == 256 and kv["dit.num_heads"] == 4
    assert kv["dit.depth"] == 3 and kv["dit.fused_depth"] == 1
    # H_ffn is read from this tensor's ne[2] (src/dit.cpp:42-43)
    assert tensors["joint_blocks.0.latent_block.ffn.w1.weight"][0] == [3, 256, 512]
    # pre_only joint block: 2H clip/text modulation, no post-attention weights
    assert tensors["joint_blocks.1.clip_block.adaLN_modulation.1.weight"][0] == [256, 512]
    assert "joint_blocks.1.clip_block.linear1.weight" not in tensors
    assert "joint_blocks.1.latent_block.linear1.weight" in tensors
    assert tensors["final_layer.conv.weight"][0] == [7, 256, 64]
    # 1-D tensors are F32 (WeightSet keeps them f32, src/net.mm:130), matrices BF16
    assert tensors["t_embed.mlp.0.bias"][1] == 0 and tensors["t_embed.mlp.0.weight"][1] == 30
    # deterministic
    p2 = str(tmp_path / "t2.gguf")
    tsn.write_synthetic_gguf(p2, make_geom(**TINY), SEED)
    assert open(p, "rb").read() == open(p2, "rb").read()
    p3 = str(tmp_path / "t3.gguf")
    tsn.write_synthetic_gguf(p3, make_geom(**TINY), SEED + 1)
    assert open(p, "rb").read() != open(p3, "rb").read()


def test_writer_rejects_unwritable_path():
    with pytest.raises(tsn.TsnError) as e:
        tsn.write_synthetic_gguf("/nonexistent-dir/x.gguf", make_geom(**TINY), SEED)
    assert e.value.code == 3
