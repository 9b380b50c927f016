"""On-device quantizers (lbc_quantize_int4 / lbc_quantize_mxfp4) against the
numpy quantizers and the reference's own packed outputs: bit for bit."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import lowbit_b200 as lb
from lowbit_b200.kernels import quantize_int4_cuda, quantize_mxfp4_cuda

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"
Z = np.load(GOLD / "golden.npz")
META = json.loads((GOLD / "golden_meta.json").read_text())
MODES = [("sym", dict()), ("asym", dict(asym=True)), ("smax", dict(scale="signed-max"))]


def host(t):
    return None if t is None else t.cpu().numpy()


def same_int4(a, b):
    np.testing.assert_array_equal(host(a.qw), b.qw)
    np.testing.assert_array_equal(host(a.scales).view(np.uint32), np.asarray(b.scales).view(np.uint32))
    if b.zeros is None:
        assert a.zeros is None
    else:
        np.testing.assert_array_equal(host(a.zeros), b.zeros)
    assert a.k == b.k


def same_mx(a, b):
    np.testing.assert_array_equal(host(a.qw), b.qw)
    np.testing.assert_array_equal(host(a.e8m0), b.e8m0)


@pytest.mark.parametrize("i", range(len(META["shapes"])))
@pytest.mark.parametrize("tag,kw", MODES)
def test_int4_matches_reference_golden(i, tag, kw):
    w = Z[f"s{i}_w"]
    q = quantize_int4_cuda(w, **kw)
    np.testing.assert_array_equal(host(q.qw), Z[f"s{i}_{tag}_qw"])
    np.testing.assert_array_equal(host(q.scales).view(np.uint32), Z[f"s{i}_{tag}_scales"].view(np.uint32))
    if tag == "asym":
        np.testing.assert_array_equal(host(q.zeros), Z[f"s{i}_{tag}_zeros"])


@pytest.mark.parametrize("i", range(len(META["shapes"])))
def test_mxfp4_matches_reference_golden(i):
    q = quantize_mxfp4_cuda(Z[f"s{i}_w"])
    np.testing.assert_array_equal(host(q.qw), Z[f"s{i}_mx_qw"])
    np.testing.assert_array_equal(host(q.e8m0), Z[f"s{i}_mx_e8m0"])


def edge_matrix():
    rng = np.random.default_rng(5)
    rows = [np.zeros(300), np.full(300, 2.5), np.full(300, -1e-3)]
    t = rng.standard_normal(300)
    t[7], t[200] = 4.0, -4.0  # signed-max tie: the first index decides the sign
    rows.append(t)
    t = rng.standard_normal(300)
    t[3], t[9] = -4.0, 4.0
    rows.append(t)
    rows.append(rng.standard_normal(300) * 1e30)
    rows.append(rng.standard_normal(300) * 1e-40)  # subnormal magnitudes
    rows.append(np.where(rng.random(300) < 0.5, -0.0, 0.0))
    rows.append(np.abs(rng.standard_normal(300)))  # all positive (asym lo = 0)
    rows.append(-np.abs(rng.standard_normal(300)))  # all negative (asym hi = 0)
    # values on E2M1 decision points after block scaling (block max 6 -> scale 1)
    grid = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.2500001, 0.7499999, 4.9999995], np.float32)
    t = np.resize(np.concatenate([grid, -grid]), 300)
    t[::32] = 6.0
    rows.append(t)
    # just below / above powers of two (block exponents)
    p = np.float32(2.0) ** rng.integers(-20, 20, 300).astype(np.float32)
    rows.append(np.nextafter(p, np.float32(0)) * np.where(rng.random(300) < 0.5, -1, 1))
    return np.asarray(rows, np.float32)


@pytest.mark.parametrize("tag,kw", MODES)
@pytest.mark.parametrize("k", [1, 31, 128, 300])
def test_int4_edge_cases_match_numpy(tag, kw, k):
    w = edge_matrix()[:, :k].copy()
    same_int4(quantize_int4_cuda(w, **kw), lb.quantize_int4(w, **kw))


@pytest.mark.parametrize("k", [1, 17, 32, 300])
def test_mxfp4_edge_cases_match_numpy(k):
    w = edge_matrix()[:, :k].copy()
    same_mx(quantize_mxfp4_cuda(w), lb.quantize_mxfp4(w))


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def test_baseline_configs_hash_to_reference():
    """The full-size BASELINE weights quantized on the GPU hash to the
    reference's packed arrays (digests recorded from lowbit itself)."""
    dig = META["digests"]
    w = torch.from_numpy(np.random.default_rng(0).standard_normal((11008, 4096)).astype(np.float32)).cuda()
    q = quantize_int4_cuda(w, asym=True)
    assert _sha(host(q.qw), host(q.scales), host(q.zeros)) == dig["w4a16_decode_packed"]
    m = quantize_mxfp4_cuda(w)
    assert _sha(host(m.qw), host(m.e8m0)) == dig["mxfp4_m64_packed"]
    w2 = np.random.default_rng(0).standard_normal((4096, 4096)).astype(np.float32)
    s = lb.quantize_int4(w2)
    same_int4(quantize_int4_cuda(w2), s)


def test_bad_arguments():
    from lowbit_b200.kernels import lib
    assert lib().lbc_quantize_int4(None, 0, 5, 0, None, None, None, None) < 0
    assert lib().lbc_quantize_int4(None, 3, 5, 1, None, None, None, None) < 0  # asym needs zeros
    assert lib().lbc_quantize_mxfp4(None, 3, 0, None, None, None) < 0
