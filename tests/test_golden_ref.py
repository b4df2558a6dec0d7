"""The CPU oracle pinned to the REFERENCE's own kernels: tests/golden/
ref_kernels.npz holds outputs of csrc/kernels.cu (compiled unmodified into
oracle/_ref/ and run on a B200 by tests/golden/make_ref_golden.py) on seeded
inputs.  No GPU needed here.

Bars: bit-exact for the codec, RMSNorm, router logits and top-k indices; the
top-k weights within rtol 1e-6 (about 8 ulp): the reference calls the device
expf (documented maximum error 2 ulp) eight times and divides by their sum,
the oracle the correctly rounded host expf.
"""
from pathlib import Path

import numpy as np
import pytest

FIX = Path(__file__).resolve().parent / "golden" / "ref_kernels.npz"


@pytest.fixture(scope="module")
def g():
    if not FIX.exists():
        pytest.skip("reference golden fixture not generated yet (tests/golden/make_ref_golden.py)")
    return dict(np.load(FIX))


def test_decode_all_codes(g, oracle):
    want = g["dequant_out"]
    got = np.array([oracle.e4m3_decode_ref(int(b)) for b in g["dequant_in"]], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_encode_reference_semantics(g, oracle):
    x, want = g["encode_in"], g["encode_out"]
    got = np.array([oracle.e4m3_encode_ref(float(v)) for v in x], dtype=np.uint8)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(float(x[i]), int(got[i]), int(want[i])) for i in bad[:10]]


@pytest.mark.parametrize("H", [512, 5120])
def test_rmsnorm_bit_exact(g, oracle, H):
    got = oracle.rmsnorm_ref(g[f"rms_x_{H}"], g[f"rms_gamma_{H}"], 1e-5)
    assert np.array_equal(got.view(np.uint32), g[f"rms_out_{H}"].view(np.uint32))


@pytest.mark.parametrize("H,E", [(512, 64), (5120, 160)])
def test_router_logits_bit_exact(g, oracle, H, E):
    got = oracle.moe_gate_ref(g[f"gate_x_{H}_{E}"], g[f"gate_w_{H}_{E}"])
    assert np.array_equal(got.view(np.uint32), g[f"gate_out_{H}_{E}"].view(np.uint32))


@pytest.mark.parametrize("name,k", [("topk", 8), ("topk2", 2)])
def test_topk(g, oracle, name, k):
    idx, w = oracle.moe_topk_ref(g[f"{name}_logits"], k)
    assert np.array_equal(idx, g[f"{name}_idx"])
    ref_w = g[f"{name}_w"]
    assert np.allclose(w, ref_w, rtol=1e-6, atol=1e-30), np.max(np.abs(w - ref_w))
