"""Failure paths on the GPU, in the forms that fault nothing.

* tsn_dit_load of a malformed or incomplete GGUF returns the code tsn_dit_inspect returns on the
  CPU (TSN_ERR_FORMAT for a bad magic or a truncated file, src/gguf.cpp:73-151; TSN_ERR_MISSING for
  an absent tensor, src/net.mm:110-118) and leaves the device usable.
* A device-side wait made to run out: the self-test kernel waits on an mbarrier nothing arrives on,
  bounded at 1 ms the way every pipeline wait of the library is bounded; the call reports
  TSN_ERR_TIMEOUT through the device error word and the context stays usable (a GEMM right after
  it is checked against float64).
"""
import numpy as np
import pytest

import tsn
from conftest import SEED, TINY, TINY_SEQ, make_geom, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    d = tsn.Device(0)
    yield d
    d.close()


def _gemm_ok(dev):
    rng = np.random.default_rng(3)
    M, N, K = 64, 256, 512
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.03).astype(np.float16)
    Y = torch.full((M, N), float("nan"), device="cuda")
    dev.gemm(True, torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda(), torch.from_numpy(x).cuda(), Y, None,
             M, N, K)
    dev.commit()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    return rel_l2(Y.cpu().numpy(), ref) < 5e-5


def _load_code(dev, path):
    with pytest.raises(tsn.TsnError) as e:
        tsn.Dit(dev, gguf=path)
    return e.value.code


def test_load_rejects_broken_files(dev, tmp_path):
    good = str(tmp_path / "good.gguf")
    tsn.write_synthetic_gguf(good, make_geom(**TINY), SEED)
    data = open(good, "rb").read()
    magic = tmp_path / "magic.gguf"
    magic.write_bytes(b"GGUX" + data[4:])
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(data[:len(data) - 1000])
    name = "final_layer.conv.weight"
    i = data.rfind(len(name).to_bytes(8, "little") + name.encode())
    missing = tmp_path / "missing.gguf"
    missing.write_bytes(data[:i + 8] + b"final_layer.conv.weighX" + data[i + 8 + len(name):])
    for path, code in ((magic, 4), (trunc, 4), (missing, 5)):
        assert _load_code(dev, str(path)) == code, path
        with pytest.raises(tsn.TsnError) as e:
            tsn.inspect(str(path))
        assert e.value.code == code
    # the device still works: a model from the good file runs a forward
    m = tsn.Dit(dev, gguf=good)
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    m.prepare(T, C, TS, 2)
    flow = np.zeros((2, T, 64), np.float32)
    m.forward(0.5, flow)
    assert np.isfinite(flow).all()
    m.close()


def test_device_wait_timeout_reports_and_recovers(dev):
    assert _gemm_ok(dev)
    for _ in range(2):
        with pytest.raises(tsn.TsnError) as e:
            dev.selftest_timeout(1000)
        assert e.value.code == 8, str(e.value)       # TSN_ERR_TIMEOUT
        assert "gave up" in str(e.value)
        assert _gemm_ok(dev), "device unusable after a bounded wait ran out"
    with pytest.raises(tsn.TsnError) as e:
        dev.selftest_timeout(5)                      # below the 100 us floor: refused on the host
    assert e.value.code == 1
