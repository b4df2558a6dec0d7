"""The serving engine's host side on CPU (include/engine.h, time_b200/engine.py,
oracle.EngineRef):

- the oracle's serving composition is invariant to where a sequence is split
  between prefill and decode (a decode step's logits equal the last row of one
  forward over the whole sequence, bit for bit) and to routing supplied back;
- init_engine reads config.json and the checkpoint of a written model and
  gets as far as device allocation (no GPU here), refuses missing or malformed
  model directories, and never crashes on them;
- the device memory plan the engine reports matches its documented layout.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from time_b200 import checkpoint as C
from time_b200 import synth

ROOT = Path(__file__).resolve().parent.parent
SHAPE = synth.TINY_MODEL


def engine_ref(oracle, w, shape, num_pages):
    layers = []
    for layer in w["layers"]:
        a = synth.attn_rank_slice(layer["attn"], shape.attn(), 1, 0)
        ffn = oracle.OracleWeights(shape.dense() if layer["dense"] else shape.moe(), layer["ffn"])
        layers.append({"attn": {k: v.cpu().numpy() for k, v in a.items()}, "ffn": ffn, "dense": layer["dense"]})
    return oracle.EngineRef(layers, w["embed"].float().numpy(), w["final_norm"].numpy(), w["lm_head"].float().numpy(),
                            shape.num_q_heads, shape.num_kv_heads, shape.rotary_dim, shape.rope_theta, shape.eps,
                            num_pages)


@pytest.fixture(scope="module")
def weights():
    return synth.make_model_weights(SHAPE, seed=5)


def test_oracle_prefill_decode_split_invariant(oracle, weights):
    rng = np.random.default_rng(0)
    L = 21
    toks = rng.integers(0, SHAPE.vocab_size, L)
    table = np.arange(4, dtype=np.int32)[None, :]           # pages 0..3 of this sequence
    # prefill positions 0..L-2, then decode position L-1
    inc = engine_ref(oracle, weights, SHAPE, 8)
    inc.forward(toks[:-1], np.arange(L - 1), np.repeat(table, L - 1, 0))
    dec = inc.forward(toks[-1:], [L - 1], table, logits=True)
    # one forward over all L positions
    full = engine_ref(oracle, weights, SHAPE, 8)
    allr = full.forward(toks, np.arange(L), np.repeat(table, L, 0), logits=True)
    assert np.array_equal(dec[0], allr[-1])
    # a second split point gives the same last-row logits too
    two = engine_ref(oracle, weights, SHAPE, 8)
    two.forward(toks[:9], np.arange(9), np.repeat(table, 9, 0))
    got = two.forward(toks[9:], np.arange(9, L), np.repeat(table, L - 9, 0), logits=True)
    assert np.array_equal(got[-1], allr[-1])


def test_oracle_supplied_routing_is_own_routing(oracle, weights):
    rng = np.random.default_rng(1)
    toks = rng.integers(0, SHAPE.vocab_size, 7)
    table = np.arange(2, dtype=np.int32)[None, :]
    a = engine_ref(oracle, weights, SHAPE, 4)
    own = []
    la = a.forward(toks, np.arange(7), np.repeat(table, 7, 0), logits=True, own_routing=own)
    routing, j = [], 0
    for layer in weights["layers"]:
        if layer["dense"]:
            routing.append(None)
        else:
            routing.append(own[j][:2])
            j += 1
    b = engine_ref(oracle, weights, SHAPE, 4)
    lb = b.forward(toks, np.arange(7), np.repeat(table, 7, 0), routing=routing, logits=True)
    assert np.array_equal(la, lb)
    assert la.shape == (7, SHAPE.vocab_size) and np.isfinite(la).all()


def _init_engine_child(model_dir: str) -> subprocess.CompletedProcess:
    code = ("import torch, sys; import time_b200.engine as E; e = E.lib(); "
            f"h = e.init_engine({model_dir!r}.encode(), 4, 64, 1); print('HANDLE', bool(h)); "
            "e.free_engine(h) if h else None")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="" if not torch.cuda.is_available() else os.environ.get(
        "CUDA_VISIBLE_DEVICES", ""))
    return subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device refusal path")
def test_init_engine_reads_model_then_needs_device(tmp_path, weights):
    C.write_model(tmp_path, SHAPE, weights, shards=2)
    r = _init_engine_child(str(tmp_path))
    assert "HANDLE False" in r.stdout, r.stdout + r.stderr
    # config and checkpoint were accepted; the refusal is the device allocation
    assert "device allocation failed" in r.stderr, r.stderr
    assert "cannot read" not in r.stderr and "unsupported" not in r.stderr


@pytest.mark.parametrize("case", ["missing_dir", "bad_json", "head_dim_64", "no_checkpoint"])
def test_init_engine_refuses_bad_model_dirs(tmp_path, weights, case):
    d = tmp_path / "m"
    if case != "missing_dir":
        C.write_model(d, SHAPE, weights)
    if case == "bad_json":
        (d / "config.json").write_text('{"hidden_size": 256,')
    elif case == "head_dim_64":
        cfg = json.loads((d / "config.json").read_text())
        cfg["head_dim"] = 64
        (d / "config.json").write_text(json.dumps(cfg))
    elif case == "no_checkpoint":
        (d / "model.safetensors").unlink()
    r = _init_engine_child(str(d))
    assert r.returncode == 0, r.stderr
    assert "HANDLE False" in r.stdout
    expect = {"missing_dir": "cannot read", "bad_json": "cannot read", "head_dim_64": "unsupported model shape",
              "no_checkpoint": "cannot open the safetensors"}[case]
    assert expect in r.stderr, r.stderr


def test_model_writer_names(weights):
    t = C.glm_model_tensors(SHAPE, weights)
    dense = [n for n in t if n.startswith("model.layers.0.mlp.")]
    assert sorted(dense) == sorted(f"model.layers.0.mlp.{p}_proj.{s}" for p in ("gate", "up", "down")
                                   for s in ("weight", "weight_scale_inv"))
    assert "model.layers.1.mlp.gate.weight" in t and "model.layers.1.mlp.shared_experts.up_proj.weight" in t
    assert t["model.embed_tokens.weight"][1].shape == (SHAPE.vocab_size, SHAPE.hidden)


@pytest.mark.parametrize("max_batch,max_seq,chunk,pages", [(4, 64, 0, 0), (64, 1024, 256, 0), (3, 100, 8, 50)])
def test_engine_device_bytes_plan(max_batch, max_seq, chunk, pages):
    """glm_engine_device_bytes = the KV pool (per layer a K and a V cache of
    [pages][16][nkv][128] bf16, 256-byte aligned), two [rows][hidden] bf16
    activation buffers (rows = max(max_batch, chunk or 2048) rounded to 16), the
    sampled rows' bf16 [max_batch][hidden], fp32 logits [max_batch][vocab], the
    page table, per-row index/weight/token arrays, a router stand-in and the
    staging block."""
    from time_b200 import engine as EN
    s = SHAPE
    got = EN.device_bytes(s, max_batch, max_seq, chunk, pages)
    rows = -(-max(max_batch, chunk or 2048) // 16) * 16
    mpps = -(-max_seq // 16)
    npages = pages or max_batch * mpps
    kv_layer = -(-(npages * 16 * s.num_kv_heads * 128 * 2) // 256) * 256
    stage = rows * (8 + 8 + 4 + 4 + 4 + 4)
    want = (kv_layer * 2 * s.num_layers + 2 * rows * s.hidden * 2 + max_batch * s.hidden * 2 +
            max_batch * s.vocab_size * 4 + max_batch * mpps * 4 + rows * (8 + 4 + 4) + s.hidden * 4 + stage)
    assert got == want, (got, want)


def test_native_engine_unloaded_behaviour(tmp_path):
    """NativeEngine before a successful load behaves as the reference's
    wrapper does (src/server/engine_wrapper.py:44-196): load() is False for a
    missing library or a model that does not load, and every call reports
    "nothing" instead of raising."""
    from time_b200 import engine as EN
    e = EN.NativeEngine(engine_path=str(tmp_path / "missing.so"), model_dir=str(tmp_path))
    assert e.load() is False and not e.is_loaded()
    e2 = EN.NativeEngine(model_dir=str(tmp_path / "no_model"))
    assert e2.load() is False and not e2.is_loaded()
    for eng in (e, e2):
        assert eng.get_info() is None
        assert eng.prefill(1, [1, 2, 3], 0.0, 1.0, 1.0, 4) is None
        assert eng.decode_step(None) == (None, True)
        assert eng.batch_decode([None, None]) == [(None, True), (None, True)]
        eng.free_request(None)
        eng.shutdown()
