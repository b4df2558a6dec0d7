"""The attention oracle (oracle/attn_oracle.c) against outputs of the
reference's own kernels (tests/golden/ref_attn.npz, written by
tests/golden/make_ref_golden.py --only attn from csrc/kernels.cu run on a
B200): paged decode attention with GQA (kernels.cu:328-392) and the KV-cache
page scatter (kernels.cu:394-410).  CPU only."""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

FIX = Path(__file__).resolve().parent / "golden" / "ref_attn.npz"


@pytest.fixture(scope="module")
def g():
    if not FIX.exists():
        pytest.skip("fixture not generated yet")
    return np.load(FIX)


@pytest.mark.parametrize("ci", [0, 1, 2, 3])
def test_oracle_attention_matches_reference_kernel(g, ci):
    nq, nkv, d, past, ps = (int(v) for v in g[f"attn{ci}_shape"])
    scale = float(g[f"attn{ci}_scale"][0])
    out = O.attn_decode_paged(g[f"attn{ci}_q"], g[f"attn{ci}_k"], g[f"attn{ci}_v"], g[f"attn{ci}_pt"], past, scale)
    ref = g[f"attn{ci}_out"]
    # the reference accumulates in fp32 (serial dot products, fp32 softmax), the oracle in double
    assert np.allclose(out, ref, rtol=2e-5, atol=2e-6), np.abs(out - ref).max()


def test_kv_scatter_layout_matches_reference(g):
    k, v, pt = g["kvw_k"], g["kvw_v"], g["kvw_pt"]
    S_, nkv, d = k.shape
    kc = np.zeros_like(g["kvw_kc"])
    vc = np.zeros_like(g["kvw_vc"])
    ps = kc.shape[1]
    for s in range(S_):
        pos = 13 + s
        kc[pt[pos // ps], pos % ps] = k[s]
        vc[pt[pos // ps], pos % ps] = v[s]
    assert np.array_equal(kc, g["kvw_kc"]) and np.array_equal(vc, g["kvw_vc"])


def test_oracle_full_rope_matches_reference_kernel():
    """rot == head_dim: the oracle's partial RoPE is the reference's rotate-half
    RoPE (fixture of tests/golden/ref_kernels.npz, kernels.cu:87-108)."""
    fix = np.load(Path(__file__).resolve().parent / "golden" / "ref_kernels.npz")
    q, qo = fix["rope_q"], fix["rope_q_out"]
    S_, NH, D = q.shape
    f = O.rope_inv_freq(D, 10000.0)
    for s in range(S_):
        got = O.rope_partial(q[s], D, 7 + s, f)
        # the reference forms its frequency with powf in fp32 and uses cosf/sinf
        assert np.allclose(got, qo[s], rtol=1e-5, atol=2e-5), np.abs(got - qo[s]).max()
