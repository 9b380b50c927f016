"""The GPU autotuner (lowbit_b200.tune, the counterpart of src/lowbit/tune.py;
the reference's tests/test_tune.py:11-30 is the model): tune a small problem,
find its entry in the cache, read it back with lookup and through
params="auto", get the same results as with the explicit tuned Params and the
oracle's within the usual bound; a cache from another GPU is ignored."""
import json

import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from lowbit_b200 import tune
from oracle import lbref as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,m", [("w4a16", 1), ("w4a16", 3), ("w4a8", 16), ("mxfp4", 1)])
def test_tune_caches_and_result_is_correct(tmp_path, monkeypatch, kind, m):
    cache = tmp_path / "tune.json"
    n, k = 512, 1024
    e = tune.tune(kind, m, n, k, reps=3, steps=8, path=cache)
    assert e["n_configs"] > 1 and e["time_s"] <= e["default_time_s"] * 1.05
    data = json.loads(cache.read_text())
    assert data["gpu"] == tune.gpu_key() and len(data["entries"]) == 1
    p = tune.lookup(kind, m, n, k, path=cache)
    assert p == K.Params(**e["params"])
    assert tune.lookup(kind, m, n, 2 * k, path=cache) is None
    rng = np.random.default_rng(0)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    W = lb.quantize_mxfp4(w) if kind == "mxfp4" else lb.quantize_int4(w)
    fn = K.GEMMS[kind]
    y = fn(x, W, p)
    # params="auto" reads the same cache entry: bit-identical results
    monkeypatch.setattr(tune, "DEFAULT_CACHE", cache)
    monkeypatch.setattr(K, "_AUTO_MEMO", {})
    real_lookup = tune.lookup
    monkeypatch.setattr(tune, "lookup", lambda *a, **kw: real_lookup(*a, path=cache))
    np.testing.assert_array_equal(fn(x, W, "auto"), y)
    if kind == "mxfp4":
        R.assert_close(y, R.gemm_mxfp4_ref(x, W.qw, W.e8m0), R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0)), 1e-5)
    elif kind == "w4a16":
        R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                       R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), 1e-5)
    else:
        a = lb.quantize_act_int8(x)
        R.assert_close(y, R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros),
                       R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros), 1e-5)


def test_tune_restricted_to_one_path(tmp_path):
    cache = tmp_path / "tune.json"
    e = tune.tune("w4a16", 1, 512, 1024, isa="mma", reps=2, steps=4, path=cache)
    assert e["params"]["isa"] == "mma"
    assert tune.lookup("w4a16", 1, 512, 1024, isa="mma", path=cache).isa == "mma"
    assert tune.lookup("w4a16", 1, 512, 1024, path=cache) is None


def test_cache_from_other_gpu_is_ignored(tmp_path):
    cache = tmp_path / "tune.json"
    cache.write_text(json.dumps({"gpu": "some other gpu", "entries": {"x": {}}}))
    assert tune.load_cache(cache)["entries"] == {}
