"""The serving engine over several GPUs of one process (glm_engine_config_t
num_gpus > 1): tensor-parallel attention (each rank its query and KV heads,
the o_proj partials summed in rank order), expert-parallel MoE layers over
NVLink peer memory on each rank's slice of the rows, the rows gathered to
every rank after each layer.  Compared with the same model on one GPU: the
logits of every decode step within the layer bar of the spec doubled for the
three-layer model (the TP sum adds the heads' partials in another order), and
bit-identical between two runs; init_engine over a written checkpoint gives
the same bits as the in-memory weights.  Needs two GPUs."""
import numpy as np
import pytest
import torch

from time_b200 import checkpoint as C
from time_b200 import engine as EN
from time_b200 import synth

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

SHAPE = synth.TINY_MODEL
MAX_REL, MAE = 2e-2, 4e-3


def to_dev(w, dev):
    if isinstance(w, torch.Tensor):
        return w.to(dev)
    if isinstance(w, dict):
        return {k: to_dev(v, dev) for k, v in w.items()}
    if isinstance(w, list):
        return [to_dev(v, dev) for v in w]
    return w


@pytest.fixture(scope="module")
def model():
    torch.cuda.set_device(0)
    w = synth.make_model_weights(SHAPE, seed=11)
    return w, to_dev(w, torch.device("cuda", 0))


def run(eng, prompts, steps):
    states = [eng.prefill(i, list(map(int, p)), 0.0, 1.0, 1.0, 32) for i, p in enumerate(prompts)]
    assert all(s is not None for s in states)
    logits, tokens = [], []
    for _ in range(steps):
        r = eng.batch_decode_raw(states)
        assert r is not None
        tokens.append([t for t, _ in r])
        logits.append(eng.copy_logits(len(prompts)))
    eng.check_error()
    return logits, tokens


def rel_mae(a, b):
    d = np.abs(a - b)
    return float(d.max() / np.abs(b).max()), float(d.mean() / np.abs(b).mean())


def test_engine_two_gpus_matches_one(model):
    _, w_dev = model
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, SHAPE.vocab_size, L) for L in (5, 17, 40)]
    one = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64)
    l1, t1 = run(one, prompts, 4)
    one.shutdown()
    two = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64, num_gpus=2)
    assert two.get_info().num_gpus == 2
    l2, t2 = run(two, prompts, 4)
    two.shutdown()
    again = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64, num_gpus=2)
    l3, t3 = run(again, prompts, 4)
    again.shutdown()
    for s in range(4):
        mr, mae = rel_mae(l2[s], l1[s])
        print(f"step {s}: two GPUs vs one: max-rel {mr:.2e} MAE {mae:.2e}; tokens {t2[s]} vs {t1[s]}")
        assert mr <= MAX_REL and mae <= MAE, (s, mr, mae)
        assert np.array_equal(l2[s], l3[s])
        assert t2[s] == t3[s]
    assert t2[0] == t1[0]


def test_engine_two_gpus_small_forwards_and_one_row(model):
    """Forwards of 8 rows (every rank's slice of the FFN rows small, a rank
    with none at a one-row decode) give the logits of one 64-row forward."""
    _, w_dev = model
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, SHAPE.vocab_size, L) for L in (21,)]
    a = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=8, num_gpus=2)
    la, ta = run(a, prompts, 3)
    a.shutdown()
    b = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64, num_gpus=2)
    lb, tb = run(b, prompts, 3)
    b.shutdown()
    for s in range(3):
        mr, mae = rel_mae(la[s], lb[s])
        assert mr <= MAX_REL and mae <= MAE, (s, mr, mae)
    assert ta[0] == tb[0]


def test_engine_two_gpus_from_checkpoint(model, tmp_path):
    w_cpu, w_dev = model
    C.write_model(tmp_path, SHAPE, w_cpu, shards=2)
    a = EN.NativeEngine(model_dir=str(tmp_path), max_batch=4, max_seq=96, num_gpus=2)
    assert a.load()
    assert a.get_info().num_gpus == 2
    b = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, num_gpus=2)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, SHAPE.vocab_size, L) for L in (9, 30)]
    la, ta = run(a, prompts, 3)
    lb, tb = run(b, prompts, 3)
    a.shutdown()
    b.shutdown()
    assert ta == tb
    for s in range(3):
        assert np.array_equal(la[s], lb[s])


def test_engine_two_gpus_decode_graphs(model, monkeypatch):
    """Decode steps replayed from per-rank CUDA graphs (the exchanges keep
    their epochs on the device) give the eager engine's logits and tokens."""
    _, w_dev = model
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, SHAPE.vocab_size, L) for L in (6, 23, 11)]
    out = {}
    for graphs in ("1", "0"):
        monkeypatch.setenv("TIME_B200_ENGINE_GRAPHS", graphs)
        eng = EN.NativeEngine.from_weights(SHAPE, w_dev, max_batch=4, max_seq=96, prefill_chunk=64, num_gpus=2)
        out[graphs] = run(eng, prompts, 6)
        eng.shutdown()
    (lg, tg), (le, te) = out["1"], out["0"]
    assert tg == te
    for a, b in zip(lg, le):
        assert np.array_equal(a, b)
