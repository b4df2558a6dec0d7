"""The serving engine on the GPU (include/engine.h through time_b200/engine.py)
against the oracle's composition of the same model (oracle.EngineRef):
prefill of several prompts, then batched decode steps, logits compared row by
row.  Each MoE layer's top-k choice is read back from the engine and given to
the oracle's expert evaluation (a near-tie in the router can flip under the
last-bit differences that several bf16 layers accumulate); the oracle's own
routing must agree except at such near-ties.  Tolerance on the fp32 logits of
the three-layer model: max |diff| / max |ref| <= 2e-2, MAE <= 4e-3 (the layer
bar of the spec, 1e-2 / 2e-3, doubled for three layers and the lm_head).

Also: the row-indexed attention block (prefill rows of one sequence next to
decode rows of another), the reference API's request semantics, init_engine
from a written checkpoint (bit-identical to the same weights in memory),
batch and prefill-chunk invariance, and top-p sampling."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from time_b200 import attn as A
from time_b200 import checkpoint as C
from time_b200 import engine as EN
from time_b200 import synth

pytestmark = pytest.mark.gpu

SHAPE = synth.TINY_MODEL
MAX_REL, MAE = 2e-2, 4e-3
PS = 16


def to_dev(w, dev):
    if isinstance(w, torch.Tensor):
        return w.to(dev)
    if isinstance(w, dict):
        return {k: to_dev(v, dev) for k, v in w.items()}
    if isinstance(w, list):
        return [to_dev(v, dev) for v in w]
    return w


def engine_ref(w, shape, num_pages):
    layers = []
    for layer in w["layers"]:
        a = synth.attn_rank_slice(layer["attn"], shape.attn(), 1, 0)
        ffn = O.OracleWeights(shape.dense() if layer["dense"] else shape.moe(), layer["ffn"])
        layers.append({"attn": {k: v.cpu().numpy() for k, v in a.items()}, "ffn": ffn, "dense": layer["dense"]})
    return O.EngineRef(layers, w["embed"].float().numpy(), w["final_norm"].numpy(), w["lm_head"].float().numpy(),
                       shape.num_q_heads, shape.num_kv_heads, shape.rotary_dim, shape.rope_theta, shape.eps, num_pages)


def gpu_routing(eng, shape, rows):
    return [None if l < shape.first_dense else eng.routing(l, rows, shape.top_k) for l in range(shape.num_layers)]


def near_tie_mismatches(gpu_r, own, shape):
    """Rows whose expert set differs between the engine and the oracle's own
    routing, and how many of them are not near-ties (gap between the k-th and
    (k+1)-th logit above 1e-3 of the row's largest logit)."""
    bad = total = 0
    j = 0
    for l in range(shape.num_layers):
        if l < shape.first_dense:
            continue
        gidx = gpu_r[l][0]
        oidx, _, lg = own[j]
        j += 1
        for r in range(gidx.shape[0]):
            if set(gidx[r]) == set(oidx[r]):
                continue
            total += 1
            s = np.sort(lg[r])[::-1]
            if s[shape.top_k - 1] - s[shape.top_k] > 1e-3 * np.abs(s).max():
                bad += 1
    return total, bad


@pytest.fixture(scope="module")
def model(gpu):
    w = synth.make_model_weights(SHAPE, seed=11)
    return w, to_dev(w, gpu)


def test_attn_block_rows_prefill_and_slots(gpu):
    """attn_block_forward over rows of two sequences: sequence in page-table
    row 1 prefills positions 0..9, the one in row 0 (context 0..4 already in
    its pages) adds positions 5..8; rows interleaved."""
    shape = synth.AttnShape(hidden=256, num_q_heads=4, num_kv_heads=2)
    rng = np.random.default_rng(3)
    w = synth.make_attn_weights(shape, seed=3, device=gpu)
    wr = synth.attn_rank_slice(w, shape, 1, 0)
    num_pages, max_pages = 6, 2
    pt = np.array([[4, 1], [0, 5]], dtype=np.int32)
    kc = torch.from_numpy(rng.standard_normal((num_pages, PS, 2, 128)).astype(np.float32)).to(torch.bfloat16).to(gpu)
    vc = torch.from_numpy(rng.standard_normal((num_pages, PS, 2, 128)).astype(np.float32)).to(torch.bfloat16).to(gpu)
    rows = [(1, p) for p in range(10)] + [(0, p) for p in range(5, 9)]
    order = rng.permutation(len(rows))
    rows = [rows[i] for i in order]
    R = len(rows)
    x = torch.from_numpy(rng.standard_normal((R, 256)).astype(np.float32)).to(torch.bfloat16).to(gpu)
    pos = torch.tensor([p for _, p in rows], dtype=torch.int32, device=gpu)
    rs = torch.tensor([s for s, _ in rows], dtype=torch.int32, device=gpu)
    blk = A.AttnBlock(shape, wr, max_batch=32, max_pages_per_seq=max_pages, max_context=max_pages * PS)
    kref, vref = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    out = blk.forward(x, pos, rs, torch.from_numpy(pt).to(gpu), kc, vc)
    blk.check_error()
    xf = x.float().cpu().numpy()
    part = O.attn_block_partial_ref({k: v.cpu().numpy() for k, v in wr.items()}, xf, [p for _, p in rows],
                                    pt[[s for s, _ in rows]], kref, vref, 4, 2, shape.rotary_dim, shape.rope_theta,
                                    shape.eps)
    ref = O.bf16_round(xf + part)
    mr, mae = O.max_rel_and_mae(out.float().cpu().numpy(), ref)
    assert mr <= 1e-2 and mae <= 2e-3, (mr, mae)
    # the K/V written for the prefilled positions match the oracle's pages
    kg = kc.float().cpu().numpy()
    for s, p in rows:
        page, slot = pt[s, p // PS], p % PS
        assert np.abs(kg[page, slot] - kref[page, slot]).max() <= 2e-2 * max(np.abs(kref[page, slot]).max(), 1)
    blk.close()


def run_parity(eng, w_cpu, prompts, steps, shape, report, rows_cap):
    """Admit `prompts`, decode `steps` batched steps; compare every step's
    logits with the oracle fed the same rows, tokens and routing.  A step's
    rows (the engine's packing): every position without K/V yet, request by
    request, then each request's newest position (the sampled rows); here
    they fit one forward (rows_cap), so the captured routing covers them."""
    P = -(-96 // PS)
    ref = engine_ref(w_cpu, shape, P * len(prompts))
    tables = [np.arange(r * P, (r + 1) * P, dtype=np.int32) for r in range(len(prompts))]
    states, toks, kv = [], [], []
    for r, pr in enumerate(prompts):
        st = eng.prefill(100 + r, list(map(int, pr)), 0.0, 1.0, 1.0, 64)
        assert st is not None
        states.append(st)
        toks.append(list(map(int, pr)))
        kv.append(0)
    ties = [0, 0]
    worst = (0.0, 0.0)
    for step in range(steps):
        rows = [(r, p) for r in range(len(toks)) for p in range(kv[r], len(toks[r]) - 1)]
        rows += [(r, len(toks[r]) - 1) for r in range(len(toks))]
        assert len(rows) <= rows_cap
        raw = eng.batch_decode_raw(states)
        R = len(states)
        lg = eng.copy_logits(R)
        rt = gpu_routing(eng, shape, len(rows))
        own = []
        lr = ref.forward([toks[r][p] for r, p in rows], [p for _, p in rows], np.stack([tables[r] for r, _ in rows]),
                         routing=rt, logits=True, own_routing=own)[-R:]
        t, b = near_tie_mismatches(rt, own, shape)
        ties[0] += t
        ties[1] += b
        mr, mae = O.max_rel_and_mae(lg, lr)
        worst = (max(worst[0], mr), max(worst[1], mae))
        for i, (tok, done) in enumerate(raw):
            assert tok == int(np.argmax(lg[i])), (step, i)     # greedy: first maximum of the engine's logits
            kv[i] = len(toks[i])
            toks[i].append(tok)
    report.update(max_rel=worst[0], mae=worst[1], routing_mismatch=ties[0], routing_mismatch_not_tie=ties[1])
    return states, toks


def test_engine_matches_oracle(gpu, model):
    w_cpu, w_dev = model
    eng = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64)
    eng.set_capture(True)
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, SHAPE.vocab_size, L) for L in (5, 17, 40)]
    rep = {}
    run_parity(eng, w_cpu, prompts, 4, SHAPE, rep, rows_cap=64)
    eng.check_error()
    print("engine vs oracle:", rep)
    assert rep["max_rel"] <= MAX_REL and rep["mae"] <= MAE, rep
    assert rep["routing_mismatch_not_tie"] == 0, rep
    eng.shutdown()


def test_engine_from_checkpoint_bit_identical(gpu, model, tmp_path):
    w_cpu, w_dev = model
    C.write_model(tmp_path, SHAPE, w_cpu, shards=3)
    a = EN.NativeEngine(model_dir=str(tmp_path), max_batch=4, max_seq=96)
    assert a.load()
    info = a.get_info()
    assert (info.hidden_dim, info.num_layers, info.num_heads, info.vocab_size, info.num_experts,
            info.top_k_experts, info.use_gpu) == (256, 3, 4, 1000, 8, 2, 1)
    assert info.num_tensors == len(C.glm_model_tensors(SHAPE, w_cpu))
    b = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96)
    rng = np.random.default_rng(8)
    prompts = [list(map(int, rng.integers(0, SHAPE.vocab_size, L))) for L in (9, 30)]
    sa = [a.prefill(i, p, 0.0, 1.0, 1.0, 16) for i, p in enumerate(prompts)]
    sb = [b.prefill(i, p, 0.0, 1.0, 1.0, 16) for i, p in enumerate(prompts)]
    for _ in range(3):
        ra, rb = a.batch_decode_raw(sa), b.batch_decode_raw(sb)
        assert ra == rb
        assert np.array_equal(a.copy_logits(2), b.copy_logits(2))
    a.shutdown()
    b.shutdown()


def test_engine_packings_match_oracle(gpu, model):
    """Request A (40-token prompt) run three ways -- alone in one forward,
    alone in forwards of at most 16 rows, and next to two other prompts in one
    forward -- each compared with the oracle's run of A alone (fed the same
    routing): the logits of its first sampled row, and every layer's K/V pages
    of its 40 positions.  The three runs are also compared with one another."""
    w_cpu, w_dev = model
    rng = np.random.default_rng(9)
    prompts = [list(map(int, rng.integers(0, SHAPE.vocab_size, L))) for L in (40, 12, 3)]
    A = prompts[0]
    variants = {"alone_one_forward": (64, [A]), "alone_16_row_forwards": (8, [A]), "batched": (64, prompts)}
    got = {}
    for name, (chunk, ps) in variants.items():
        eng = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=chunk)
        eng.set_capture(True)
        st = [eng.prefill(i, p, 0.0, 1.0, 1.0, 16) for i, p in enumerate(ps)]
        eng.batch_decode_raw(st)
        # the step's rows: prompts' positions 0..L-2 request by request, then the sampled rows
        rows = [(i, q) for i, p in enumerate(ps) for q in range(len(p) - 1)] + [(i, len(p) - 1) for i, p in enumerate(ps)]
        sel = [j for j, (i, _) in enumerate(rows) if i == 0]          # A's rows, positions 0..39
        routing = []
        for l in range(SHAPE.num_layers):
            if l < SHAPE.first_dense:
                routing.append(None)
            else:
                idx, w = eng.routing(l, len(rows), SHAPE.top_k)
                routing.append((idx[sel], w[sel]))
        pages = eng.request_pages(st[0])
        kv = [eng.kv_pages(l, pages, SHAPE.num_kv_heads) for l in range(SHAPE.num_layers)]
        got[name] = (eng.copy_logits(len(ps))[0], routing, kv)
        eng.check_error()
        eng.shutdown()
    report = {}
    for name, (lg, routing, kv) in got.items():
        ref = engine_ref(w_cpu, SHAPE, 8)
        table = np.arange(3, dtype=np.int32)[None]
        lr = ref.forward(A, np.arange(40), np.repeat(table, 40, 0), routing=routing, logits=True)[-1]
        mr, mae = O.max_rel_and_mae(lg, lr)
        kvd = []
        for l in range(SHAPE.num_layers):
            k, v = kv[l]
            kr = ref.k[l][:3].reshape(48, SHAPE.num_kv_heads, 128)[:40]
            vr = ref.v[l][:3].reshape(48, SHAPE.num_kv_heads, 128)[:40]
            kg = k.reshape(48, SHAPE.num_kv_heads, 128)[:40]
            vg = v.reshape(48, SHAPE.num_kv_heads, 128)[:40]
            kvd.append((float(np.abs(kg - kr).max() / np.abs(kr).max()), float(np.abs(vg - vr).max() / np.abs(vr).max())))
        report[name] = {"logits_max_rel": mr, "logits_mae": mae, "kv_max_rel_per_layer": kvd}
    names = list(got)
    for a_, b_ in ((names[0], names[1]), (names[0], names[2])):
        report[f"{a_}=={b_}"] = {"logits": bool(np.array_equal(got[a_][0], got[b_][0])),
                                 "kv": [bool(np.array_equal(got[a_][2][l][0], got[b_][2][l][0])) and
                                        bool(np.array_equal(got[a_][2][l][1], got[b_][2][l][1]))
                                        for l in range(SHAPE.num_layers)]}
    print("packings:", report)
    for name in got:
        r = report[name]
        assert r["logits_max_rel"] <= MAX_REL and r["logits_mae"] <= MAE, (name, r)
        assert all(k <= 2e-2 and v <= 2e-2 for k, v in r["kv_max_rel_per_layer"]), (name, r)


def test_engine_two_engines_from_one_weight_dict(gpu, model):
    """Two engines alive at once over the same weights dict (each makes its
    own rank-layout attention copies and keeps them): request A alone in
    16-row forwards and A next to two other prompts give bit-identical
    logits at every step."""
    _, w_dev = model
    rng = np.random.default_rng(9)
    prompts = [list(map(int, rng.integers(0, SHAPE.vocab_size, L))) for L in (40, 12, 3)]
    e1 = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=8)
    e3 = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64)
    s1 = e1.prefill(0, prompts[0], 0.0, 1.0, 1.0, 16)
    s3 = [e3.prefill(i, p, 0.0, 1.0, 1.0, 16) for i, p in enumerate(prompts)]
    for _ in range(3):
        t1 = e1.decode_step(s1)
        r3 = e3.batch_decode_raw(s3)
        assert np.array_equal(e1.copy_logits(1)[0], e3.copy_logits(3)[0])
        assert t1[0] == r3[0][0]
    e1.shutdown()
    e3.shutdown()


def test_engine_request_semantics(gpu, model):
    _, w_dev = model
    # 3 KV pages in all: a 40-token prompt holds all three (positions 0..47)
    eng = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=2, max_seq=64, num_cache_pages=3)
    info = eng.get_info()
    assert (info.kv_pages_max, info.kv_pages_used, info.active_requests, info.max_batch, info.max_seq) == (3, 0, 0, 2,
                                                                                                         64)
    rng = np.random.default_rng(10)
    assert eng.prefill(1, [5] * 65, 0.0, 1.0, 1.0, 4) is None          # longer than max_seq
    assert eng.prefill(1, [], 0.0, 1.0, 1.0, 4) is None
    assert eng.prefill(1, [SHAPE.vocab_size], 0.0, 1.0, 1.0, 4) is None  # token outside the vocabulary
    a = eng.prefill(1, list(map(int, rng.integers(0, SHAPE.vocab_size, 40))), 0.0, 1.0, 1.0, 20)
    assert a is not None and eng.get_info().kv_pages_used == 3
    assert eng.prefill(2, [1, 2], 0.0, 1.0, 1.0, 4) is None             # no KV page left
    # positions 39..47 fit the three pages; position 48 needs a fourth: the request ends there
    outs = [eng.decode_step(a) for _ in range(10)]
    assert all(not d for _, d in outs[:9]) and outs[9] == (None, True)
    eng.free_request(a)
    assert eng.get_info().kv_pages_used == 0 and eng.get_info().active_requests == 0
    # max_tokens: done with the max_tokens-th token
    b = eng.prefill(3, [1, 2, 3], 0.0, 1.0, 1.0, 2)
    c = eng.prefill(4, [4], 0.0, 1.0, 1.0, 3)
    r1 = eng.batch_decode_raw([b, c, None])
    assert [d for _, d in r1] == [False, False, True] and r1[2][0] == 0
    r2 = eng.batch_decode_raw([b, c])
    assert [d for _, d in r2] == [True, False]
    r3 = eng.batch_decode_raw([b, c])
    assert r3[0] == (0, True) and r3[1][1] is True
    assert eng.batch_decode([b, c]) == [(None, True), (None, True)]
    assert eng.prefill(5, [1], 0.0, 1.0, 1.0, 2) is None                # both request slots in use
    eng.free_request(b)
    eng.free_request(c)
    eng.check_error()
    eng.shutdown()


def test_engine_top_p_sampling(gpu, model):
    """temperature 0.8, top_p 0.9: the token is where the reference's CDF
    inversion lands on the engine's own logits (kernels.cu:236-262) with the
    reference's seed (engine.t:1446-1448)."""
    _, w_dev = model
    eng = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96)
    rng = np.random.default_rng(12)
    ids = [7, 8, 9]
    prompts = [list(map(int, rng.integers(0, SHAPE.vocab_size, L))) for L in (6, 11, 2)]
    states = [eng.prefill(i, p, 0.8, 0.9, 1.0, 8) for i, p in zip(ids, prompts)]
    past = [len(p) for p in prompts]
    for _ in range(3):
        raw = eng.batch_decode_raw(states)
        lg = eng.copy_logits(3).astype(np.float64)
        for i, (tok, _) in enumerate(raw):
            seed = ((ids[i] * 31 + past[i] * 17) * 6364136223846793005 + 1442695040888963407) % (1 << 64)
            rv = np.float32(seed & 0xFFFFFFFF) / np.float32(4294967296.0)
            e = np.exp((lg[i] - lg[i].max()) / 0.8)
            cum = np.cumsum(e)
            target = float(rv) * 0.9 * cum[-1]
            lo = cum[tok - 1] if tok > 0 else 0.0
            assert lo <= target * (1 + 1e-4) and cum[tok] >= target * (1 - 1e-4), (i, tok)
            past[i] += 1
    eng.shutdown()


def test_engine_decode_graphs_bit_identical(gpu, model, monkeypatch):
    """Pure decode steps replay a CUDA graph of the whole forward (captured
    the second time a row count occurs): logits and tokens of six steps equal
    the eager engine's (TIME_B200_ENGINE_GRAPHS=0), including after a request
    finishes and the row count changes."""
    _, w_dev = model
    rng = np.random.default_rng(12)
    prompts = [list(map(int, rng.integers(0, SHAPE.vocab_size, L))) for L in (7, 19, 33)]

    def run(graphs):
        monkeypatch.setenv("TIME_B200_ENGINE_GRAPHS", "1" if graphs else "0")
        eng = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64)
        st = [eng.prefill(i, p, 0.0, 1.0, 1.0, 4 if i == 1 else 16) for i, p in enumerate(prompts)]
        out = []
        finished = [False] * len(st)
        for _ in range(6):
            rows = finished.count(False)          # rows of this step: the requests not finished before it
            r = eng.batch_decode_raw(st)
            out.append(([t for t, _ in r], eng.copy_logits(rows)))
            finished = [f or d for f, (_, d) in zip(finished, r)]
        eng.check_error()
        eng.shutdown()
        return out
    a, b = run(True), run(False)
    for (ta, la), (tb, lb) in zip(a, b):
        assert ta == tb
        assert np.array_equal(la, lb)
