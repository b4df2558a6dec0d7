"""The safetensors loader (include/st_loader.h, time_b200/checkpoint.py) on
CPU: checkpoints written from this package's synthetic weights (single file
and index + shards, HF GLM-4.x names) read back tensor by tensor, assembled
into MoELayer's layout (EP slices, expert placement) and AttnBlock's rank
layout and compared with synth's own layouts; bf16/f16 conversions checked
against torch; malformed files refused with an error code."""
import json
import struct

import numpy as np
import pytest
import torch

from time_b200 import checkpoint as C
from time_b200 import moe as M
from time_b200 import synth

SHAPE = synth.MoEShape(hidden=256, num_experts=8, top_k=2, intermediate=256, num_shared=1)
ASHAPE = synth.AttnShape(hidden=256, num_q_heads=4, num_kv_heads=2)


@pytest.fixture(scope="module")
def weights():
    w = synth.make_moe_weights(SHAPE, seed=3, zipf_bias=True)
    a = synth.make_attn_weights(ASHAPE, seed=4)
    a["gamma"] = torch.linspace(0.5, 1.5, ASHAPE.hidden)
    w["gamma"] = torch.linspace(-1.0, 1.0, SHAPE.hidden)
    return w, a


@pytest.mark.parametrize("shards", [1, 3])
def test_round_trip_tensors(tmp_path, weights, shards):
    w, a = weights
    t = C.glm_tensors_from_synth(w, SHAPE, layer=2, attn_w=a, router_dtype="F32", norm_dtype="F32")
    C.write_checkpoint(tmp_path, t, shards=shards)
    with C.Checkpoint(tmp_path) as ck:
        assert sorted(ck.names()) == sorted(t)
        for name, (dt, arr) in t.items():
            gdt, got = ck.get(name)
            assert gdt == dt and got.shape == arr.shape and np.array_equal(got.view(np.uint8), arr.view(np.uint8))


def test_single_file_path(tmp_path, weights):
    w, _ = weights
    t = C.glm_tensors_from_synth(w, SHAPE, layer=0, router_dtype="F32", norm_dtype="F32")
    C.write_safetensors(tmp_path / "x.safetensors", t, metadata={"format": "pt"})
    with C.Checkpoint(tmp_path / "x.safetensors") as ck:
        assert len(ck.names()) == len(t)


@pytest.mark.parametrize("ep,rank,placed", [(1, 0, False), (2, 1, False), (2, 0, True), (4, 3, True)])
def test_moe_layer_layout(tmp_path, weights, ep, rank, placed):
    w, _ = weights
    t = C.glm_tensors_from_synth(w, SHAPE, layer=5, router_dtype="F32", norm_dtype="F32")
    C.write_checkpoint(tmp_path, t, shards=2)
    placement = None
    if placed:
        placement = np.random.default_rng(ep + rank).permutation(SHAPE.num_experts).astype(np.int32).tolist()
    with C.Checkpoint(tmp_path) as ck:
        got = ck.moe_layer("model.layers.5.", SHAPE, ep_size=ep, ep_rank=rank, placement=placement)
    ref = synth.expert_slice(w, SHAPE, ep, rank, slot_of_expert=placement) if ep > 1 else w
    for k in ("w13", "s13", "w2", "s2"):
        assert torch.equal(got[k], ref[k]), k
    assert torch.equal(got["router_w"], w["router_w"]) and torch.equal(got["gamma"], w["gamma"])
    assert torch.equal(got["router_bias"], w["router_bias"])


def test_bf16_and_f16_conversion(tmp_path, weights):
    w, a = weights
    t = C.glm_tensors_from_synth(w, SHAPE, layer=1, attn_w=a, router_dtype="BF16", norm_dtype="F16")
    del t["model.layers.1.mlp.gate.e_score_correction_bias"]
    C.write_checkpoint(tmp_path, t)
    with C.Checkpoint(tmp_path) as ck:
        got = ck.moe_layer("model.layers.1.", SHAPE)
        att = ck.attn_rank("model.layers.1.", ASHAPE)
    assert got["router_bias"] is None
    assert torch.equal(got["router_w"], w["router_w"].to(torch.bfloat16).float())
    assert torch.equal(got["gamma"], w["gamma"].to(torch.float16).float())
    assert torch.equal(att["gamma"], a["gamma"].to(torch.float16).float())


@pytest.mark.parametrize("tp,rank", [(1, 0), (2, 0), (2, 1)])
def test_attn_rank_layout(tmp_path, weights, tp, rank):
    w, a = weights
    t = C.glm_tensors_from_synth(w, SHAPE, layer=7, attn_w=a, norm_dtype="F32")
    C.write_checkpoint(tmp_path, t, shards=2)
    with C.Checkpoint(tmp_path) as ck:
        got = ck.attn_rank("model.layers.7.", ASHAPE, tp=tp, rank=rank)
    ref = synth.attn_rank_slice(a, ASHAPE, tp, rank)
    for k in ("w_qkv", "s_qkv", "w_o", "s_o", "gamma"):
        assert torch.equal(got[k], ref[k]), k


def _raw(path, header: bytes, data: bytes = b"", hlen=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header) if hlen is None else hlen))
        f.write(header)
        f.write(data)


@pytest.mark.parametrize("case", ["bad_json", "offsets_past_end", "size_mismatch", "unknown_dtype", "header_past_end",
                                  "duplicate", "short_file", "missing_in_shard", "shard_outside_dir", "no_files"])
def test_malformed_refused(tmp_path, case):
    f = tmp_path / "model.safetensors"
    ok_hdr = {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}
    if case == "bad_json":
        _raw(f, b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]', b"\0" * 8)
    elif case == "offsets_past_end":
        _raw(f, json.dumps({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}).encode(), b"\0" * 4)
    elif case == "size_mismatch":
        _raw(f, json.dumps({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}).encode(), b"\0" * 8)
    elif case == "unknown_dtype":
        _raw(f, json.dumps({"a": {"dtype": "Q4", "shape": [2], "data_offsets": [0, 8]}}).encode(), b"\0" * 8)
    elif case == "header_past_end":
        _raw(f, json.dumps(ok_hdr).encode(), b"\0" * 8, hlen=10 ** 6)
    elif case == "duplicate":
        _raw(f, b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}, '
                b'"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}', b"\0" * 8)
    elif case == "short_file":
        f.write_bytes(b"\1\2\3")
    elif case in ("missing_in_shard", "shard_outside_dir"):
        _raw(tmp_path / "s1.safetensors", json.dumps(ok_hdr).encode(), b"\0" * 8)
        shard = "s1.safetensors" if case == "missing_in_shard" else "../s1.safetensors"
        (tmp_path / "model.safetensors.index.json").write_text(
            json.dumps({"weight_map": {"a": shard, "b": shard}}))
    else:
        pass   # empty directory
    with pytest.raises(M.MoEError) as e:
        C.Checkpoint(tmp_path)
    assert e.value.code in (1, 3)


def test_missing_layer_tensor_refused(tmp_path, weights):
    w, _ = weights
    t = C.glm_tensors_from_synth(w, SHAPE, layer=0, router_dtype="F32")
    del t["model.layers.0.mlp.experts.3.down_proj.weight_scale_inv"]
    C.write_checkpoint(tmp_path, t)
    with C.Checkpoint(tmp_path) as ck:
        ck.moe_layer("model.layers.0.", SHAPE, ep_size=2, ep_rank=1)       # experts 4-7: fine
        with pytest.raises(M.MoEError):
            ck.moe_layer("model.layers.0.", SHAPE, ep_size=2, ep_rank=0)
