"""Seeded synthetic inputs for the MoE FFN block (shapes of BASELINE.json's
configurations), generated with torch so the same code runs on the CPU (small
parity cases) and on the GPU (full-size benchmark weights).

Draw order for one seed: x, router weight, router bias permutation, then for
every expert e = 0..E-1 its gate, up and down matrices, then the shared
expert.  Weights ~ N(0, 0.02) are quantised to E4M3 per 128x128 block with
scale = amax / 448 (q = rne(w * 448/amax)); the zipf bias is
b_e = -1.1 * ln(pi_e) for a seeded permutation pi of 1..E.
"""
from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class MoEShape:
    hidden: int
    num_experts: int
    top_k: int
    intermediate: int
    num_shared: int = 1
    eps: float = 1e-5

    @property
    def groups(self) -> int:
        return self.num_experts + self.num_shared


# BASELINE.json configs[0] (tiny CPU layer) and configs[1] (GLM-4.x MoE FFN)
TINY = MoEShape(hidden=256, num_experts=8, top_k=2, intermediate=512, num_shared=1, eps=1e-5)
GLM = MoEShape(hidden=5120, num_experts=160, top_k=8, intermediate=1536, num_shared=1, eps=1e-5)


def quantize_blocks(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[rows][cols] fp32 -> (e4m3 bytes [rows][cols] uint8, scales [rows/128][cols/128] fp32)."""
    rows, cols = w.shape
    assert rows % 128 == 0 and cols % 128 == 0
    blk = w.reshape(rows // 128, 128, cols // 128, 128)
    amax = blk.abs().amax(dim=(1, 3))                      # [rb][cb]
    safe = torch.where(amax > 0, amax, torch.ones_like(amax))
    inv = torch.where(amax > 0, 448.0 / safe, torch.zeros_like(amax))
    q = (blk * inv[:, None, :, None]).reshape(rows, cols).to(torch.float8_e4m3fn)
    scale = torch.where(amax > 0, amax / 448.0, torch.zeros_like(amax)).to(torch.float32)
    return q.view(torch.uint8), scale.contiguous()


def make_moe_weights(shape: MoEShape, seed: int = 0, device="cpu", zipf_bias: bool = False,
                     gen: torch.Generator | None = None, skip_x: bool = True, experts: bool = True) -> dict:
    """Router + expert weights (see module docstring for the draw order).
    experts=False stops after the router (gamma, router_w, router_bias: the
    same values as the full draw)."""
    g = gen or torch.Generator(device=device).manual_seed(seed)
    H, E, I, S = shape.hidden, shape.num_experts, shape.intermediate, shape.num_shared
    out = {"gamma": torch.ones(H, dtype=torch.float32, device=device)}
    out["router_w"] = torch.randn(E, H, generator=g, device=device, dtype=torch.float32) * 0.02
    if zipf_bias:
        perm = torch.randperm(E, generator=g, device=device).to(torch.float32) + 1.0
        out["router_bias"] = (-1.1 * torch.log(perm)).to(torch.float32)
    else:
        out["router_bias"] = None
    if not experts:
        return out
    G = E + S
    w13 = torch.empty(G, 2 * I, H, dtype=torch.uint8, device=device)
    s13 = torch.empty(G, 2 * I // 128, H // 128, dtype=torch.float32, device=device)
    w2 = torch.empty(G, H, I, dtype=torch.uint8, device=device)
    s2 = torch.empty(G, H // 128, I // 128, dtype=torch.float32, device=device)
    for e in range(G):
        gate = torch.randn(I, H, generator=g, device=device, dtype=torch.float32) * 0.02
        up = torch.randn(I, H, generator=g, device=device, dtype=torch.float32) * 0.02
        down = torch.randn(H, I, generator=g, device=device, dtype=torch.float32) * 0.02
        q, s = quantize_blocks(torch.cat([gate, up], 0))
        w13[e].copy_(q)
        s13[e].copy_(s)
        q, s = quantize_blocks(down)
        w2[e].copy_(q)
        s2[e].copy_(s)
    out.update(w13=w13, s13=s13, w2=w2, s2=s2)
    return out


def expert_slice(w: dict, shape: MoEShape, ep_size: int, ep_rank: int, slot_of_expert=None) -> dict:
    """The weights expert-parallel rank `ep_rank` holds: its routed experts in
    local-slot order -- [r*E/ep, (r+1)*E/ep) for the contiguous placement, or
    the experts whose slot (slot_of_expert[e]) lies in that range -- then the
    shared expert(s), as contiguous copies; the router stays replicated."""
    E, S = shape.num_experts, shape.num_shared
    per = E // ep_size
    if slot_of_expert is None:
        routed = list(range(ep_rank * per, (ep_rank + 1) * per))
    else:
        by_slot = sorted(range(E), key=lambda e: int(slot_of_expert[e]))
        routed = by_slot[ep_rank * per:(ep_rank + 1) * per]
    keep = routed + list(range(E, E + S))
    out = {k: v for k, v in w.items() if k not in ("w13", "s13", "w2", "s2")}
    for k in ("w13", "s13", "w2", "s2"):
        out[k] = w[k][keep].contiguous()
    return out


def token_slice(tokens: int, ep_size: int, ep_rank: int) -> tuple[int, int]:
    """[begin, end) of the global tokens rank `ep_rank` owns (contiguous,
    the first tokens % ep_size ranks one longer)."""
    base, extra = divmod(tokens, ep_size)
    begin = ep_rank * base + min(ep_rank, extra)
    return begin, begin + base + (1 if ep_rank < extra else 0)


def make_x(shape: MoEShape, tokens: int, seed: int = 0, device="cpu",
           gen: torch.Generator | None = None) -> torch.Tensor:
    g = gen or torch.Generator(device=device).manual_seed(seed)
    return torch.randn(tokens, shape.hidden, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


def make_case(shape: MoEShape, tokens: int, seed: int = 0, device="cpu", zipf_bias: bool = False) -> dict:
    """x then weights from one generator (the documented draw order)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = make_x(shape, tokens, device=device, gen=g)
    w = make_moe_weights(shape, device=device, zipf_bias=zipf_bias, gen=g)
    w["x"] = x
    return w


def zipf_bias(E: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(E, generator=g).to(torch.float32) + 1.0
    return (-1.1 * torch.log(perm)).to(torch.float32)


def uniform_routing(tokens: int, E: int, k: int, seed: int = 0, device="cpu"):
    """Router logits ~ U(0,1) [T][E]; returns the logits."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.rand(tokens, E, generator=g, device=device, dtype=torch.float32)


def expected_distinct_ranks(E: int, k: int, ep: int) -> float:
    """Mean number of distinct EP ranks a token's k experts land on."""
    per = E // ep
    return ep * (1.0 - math.comb(E - per, k) / math.comb(E, k))


def balanced_placement(expert_load, ep_size: int) -> list[int]:
    """Expert -> slot permutation that evens the ranks' expected work
    (longest-processing-time first: heaviest expert to the least loaded rank
    that still has a free slot; every rank gets E/ep experts, in ascending
    expert order within the rank).  `expert_load`: per-expert routed pairs
    measured on a calibration batch."""
    load = [float(v) for v in expert_load]
    E = len(load)
    per = E // ep_size
    owner = [0] * E
    rank_load = [0.0] * ep_size
    rank_n = [0] * ep_size
    for e in sorted(range(E), key=lambda i: (-load[i], i)):
        r = min((r for r in range(ep_size) if rank_n[r] < per), key=lambda r: (rank_load[r], r))
        owner[e] = r
        rank_load[r] += load[e]
        rank_n[r] += 1
    slot = [0] * E
    for r in range(ep_size):
        mine = sorted(e for e in range(E) if owner[e] == r)
        for j, e in enumerate(mine):
            slot[e] = r * per + j
    return slot


# ---------------------------------------------------------------- attention block (config 4)

@dataclasses.dataclass(frozen=True)
class AttnShape:
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int = 128
    rotary_dim: int = 64
    rope_theta: float = 1e6
    eps: float = 1e-5


# GLM-4.x attention, TP = 8 (12 query heads and 1 KV head per rank)
GLM_ATTN = AttnShape(hidden=5120, num_q_heads=96, num_kv_heads=8)


def make_attn_weights(shape: AttnShape, seed: int = 0, device="cpu") -> dict:
    """Whole-model q/k/v/o projections ~N(0, 0.02) quantised per 128x128 block,
    gamma = 1 (draw order: q, k, v, o)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, d = shape.hidden, shape.head_dim
    out = {"gamma": torch.ones(H, dtype=torch.float32, device=device)}
    for name, rows, cols in (("q", shape.num_q_heads * d, H), ("k", shape.num_kv_heads * d, H),
                             ("v", shape.num_kv_heads * d, H), ("o", H, shape.num_q_heads * d)):
        w = torch.randn(rows, cols, generator=g, device=device, dtype=torch.float32) * 0.02
        out["w_" + name], out["s_" + name] = quantize_blocks(w)
    return out


def attn_rank_slice(w: dict, shape: AttnShape, tp: int, rank: int) -> dict:
    """Rank `rank`'s weights: its query heads [r*nq/tp, (r+1)*nq/tp) and KV heads
    (shard_heads, kernels.fut:619-630) stacked q, k, v for the QKV projection,
    and the matching input columns of o_proj (row-parallel)."""
    d = shape.head_dim
    nq, nkv = shape.num_q_heads // tp, shape.num_kv_heads // tp
    q_rows = slice(rank * nq * d, (rank + 1) * nq * d)
    kv_rows = slice(rank * nkv * d, (rank + 1) * nkv * d)
    qb, kb = slice(rank * nq * d // 128, (rank + 1) * nq * d // 128), slice(rank * nkv * d // 128, (rank + 1) * nkv * d // 128)
    return {
        "gamma": w["gamma"],
        "w_qkv": torch.cat([w["w_q"][q_rows], w["w_k"][kv_rows], w["w_v"][kv_rows]]).contiguous(),
        "s_qkv": torch.cat([w["s_q"][qb], w["s_k"][kb], w["s_v"][kb]]).contiguous(),
        "w_o": w["w_o"][:, q_rows].contiguous(),
        "s_o": w["s_o"][:, qb].contiguous(),
    }



# ---------------------------------------------------------------- whole model (serving)

@dataclasses.dataclass(frozen=True)
class ModelShape:
    """A GLM-4.x decoder: `first_dense` dense-FFN layers, then MoE layers."""
    hidden: int
    num_layers: int
    first_dense: int
    num_q_heads: int
    num_kv_heads: int
    vocab_size: int
    num_experts: int
    top_k: int
    moe_intermediate: int
    num_shared: int
    dense_intermediate: int
    head_dim: int = 128
    rotary_dim: int = 64
    rope_theta: float = 1e6
    eps: float = 1e-5

    def attn(self) -> AttnShape:
        return AttnShape(self.hidden, self.num_q_heads, self.num_kv_heads, self.head_dim, self.rotary_dim,
                         self.rope_theta, self.eps)

    def moe(self) -> MoEShape:
        return MoEShape(self.hidden, self.num_experts, self.top_k, self.moe_intermediate, self.num_shared, self.eps)

    def dense(self) -> MoEShape:
        """The dense FFN as a one-expert MoE layer (weight 1.0, no shared expert)."""
        return MoEShape(self.hidden, 1, 1, self.dense_intermediate, 0, self.eps)


TINY_MODEL = ModelShape(hidden=256, num_layers=3, first_dense=1, num_q_heads=4, num_kv_heads=2, vocab_size=1000,
                        num_experts=8, top_k=2, moe_intermediate=256, num_shared=1, dense_intermediate=512)
# 92 layers, the first 3 dense (I = 12288), vocabulary 151552
GLM_MODEL = ModelShape(hidden=5120, num_layers=92, first_dense=3, num_q_heads=96, num_kv_heads=8,
                       vocab_size=151552, num_experts=160, top_k=8, moe_intermediate=1536, num_shared=1,
                       dense_intermediate=12288)


def make_model_weights(shape: ModelShape, seed: int = 0, device="cpu", share_layers: bool = False) -> dict:
    """Embedding bf16 [V][H] ~ N(0, 1), lm_head bf16 ~ N(0, 0.02), final-norm
    and per-layer RMSNorm gammas 1 + 0.1 N(0, 1), and per layer the attention
    (make_attn_weights) and FFN (make_moe_weights; the dense layers as one
    expert) weights: layer l's projections from seed * 1000 + l + 1, its
    gammas and FFN from a generator seeded seed * 1000 + 500 + l.  share_layers: one attention, one dense and one MoE weight set
    reused by every layer (a whole-depth model in one GPU's memory for
    timing; each layer still reads its full weights from HBM)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, V = shape.hidden, shape.vocab_size
    out = {
        "embed": torch.randn(V, H, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16),
        "lm_head": (torch.randn(V, H, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16),
        "final_norm": 1.0 + 0.1 * torch.randn(H, generator=g, device=device, dtype=torch.float32),
    }
    layers = []
    cache = {}
    for l in range(shape.num_layers):
        dense = l < shape.first_dense
        key = "dense" if dense else "moe"
        if share_layers and key in cache:
            layers.append(cache[key])
            continue
        lg = torch.Generator(device=device).manual_seed(seed * 1000 + 500 + l)
        attn = make_attn_weights(shape.attn(), seed=seed * 1000 + l + 1, device=device)
        attn["gamma"] = 1.0 + 0.1 * torch.randn(H, generator=lg, device=device, dtype=torch.float32)
        ffn = make_moe_weights(shape.dense() if dense else shape.moe(), device=device, gen=lg)
        ffn["gamma"] = 1.0 + 0.1 * torch.randn(H, generator=lg, device=device, dtype=torch.float32)
        entry = {"attn": attn, "ffn": ffn, "dense": dense}
        cache[key] = entry
        layers.append(entry)
    out["layers"] = layers
    return out
