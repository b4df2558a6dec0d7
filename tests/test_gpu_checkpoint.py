"""A layer loaded from a safetensors checkpoint (time_b200/checkpoint.py)
computes the same bits as the layer built from the weights it was written
from: the MoE layer (with an expert-parallel slice and placement assembled by
the loader, run as the emulated EP forward's building block) and the decode
attention block."""
import numpy as np
import pytest
import torch

from time_b200 import attn as A
from time_b200 import checkpoint as C
from time_b200 import moe as M
from time_b200 import synth

pytestmark = pytest.mark.gpu


def test_moe_layer_from_checkpoint_bit_identical(gpu, tmp_path):
    shape = synth.TINY
    w = synth.make_moe_weights(shape, seed=2, zipf_bias=True)
    C.write_checkpoint(tmp_path, C.glm_tensors_from_synth(w, shape, layer=4, router_dtype="F32", norm_dtype="F32"),
                       shards=2)
    x = synth.make_x(shape, 64, seed=5).to(gpu)
    ref_layer = M.MoELayer(shape, {k: (v.to(gpu) if isinstance(v, torch.Tensor) else v) for k, v in w.items()},
                           max_tokens=64)
    ref = ref_layer.forward(x)
    with C.Checkpoint(tmp_path) as ck:
        lw = ck.moe_layer("model.layers.4.", shape, device=gpu)
    layer = M.MoELayer(shape, lw, max_tokens=64)
    out = layer.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    layer.close()
    ref_layer.close()


def test_attn_block_from_checkpoint_bit_identical(gpu, tmp_path):
    ashape = synth.AttnShape(hidden=512, num_q_heads=8, num_kv_heads=2)
    mshape = synth.MoEShape(hidden=512, num_experts=2, top_k=1, intermediate=128)
    a = synth.make_attn_weights(ashape, seed=6)
    w = synth.make_moe_weights(mshape, seed=7)
    C.write_checkpoint(tmp_path, C.glm_tensors_from_synth(w, mshape, layer=0, attn_w=a, norm_dtype="F32"))
    rng = np.random.default_rng(1)
    tp, rank = 2, 1
    kc = torch.from_numpy(rng.standard_normal((6, 16, 1, 128)).astype(np.float32)).to(torch.bfloat16).to(gpu)
    vc = torch.from_numpy(rng.standard_normal((6, 16, 1, 128)).astype(np.float32)).to(torch.bfloat16).to(gpu)
    x = torch.from_numpy(rng.standard_normal((2, 512)).astype(np.float32)).to(torch.bfloat16).to(gpu)
    pos = torch.tensor([17, 40], dtype=torch.int32, device=gpu)
    pt = torch.tensor([[0, 1, -1], [2, 3, 4]], dtype=torch.int32, device=gpu)
    outs = []
    with C.Checkpoint(tmp_path) as ck:
        sources = [synth.attn_rank_slice(a, ashape, tp, rank), ck.attn_rank("model.layers.0.", ashape, tp=tp, rank=rank)]
    for wr in sources:
        blk = A.AttnBlock(ashape, {k: v.to(gpu) for k, v in wr.items()}, max_batch=2, max_pages_per_seq=3,
                          max_context=48, tp_size=tp, tp_rank=rank)
        outs.append(blk.decode_partial(x, pos, pt, kc.clone(), vc.clone()))
        torch.cuda.synchronize()
        blk.check_error()
        blk.close()
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
