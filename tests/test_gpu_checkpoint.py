"""On-device restore of a quantized checkpoint: bytes land unchanged in GPU memory
(through small staging chunks, so tensors span several chunks), the packed experts
come back as kernel-ready handles, and a PACKED model restored from disk computes
the same layer as the one that was saved."""

from __future__ import annotations

import json
import os

import pytest
import torch
from safetensors.torch import load_file, save_file

pytestmark = pytest.mark.gpu


def _model_and_checkpoint(tmp_path):
    from llada_quant_b200 import symmetric as G
    from llada_quant_b200.moe import QuantExpertWeights, attach_packed_buffers, install_packed_expert_access
    E, H, I = 8, 1024, 512
    g = torch.Generator(device="cuda").manual_seed(0)
    blocks = torch.nn.Module()
    b = torch.nn.Module()
    b.w1 = torch.nn.Parameter((torch.randn(E, 2 * I, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
    b.w2 = torch.nn.Parameter((torch.randn(E, H, I, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
    blocks.add_module("0", b)
    model = torch.nn.Module()
    model.add_module("blocks", blocks)
    model.gate = torch.nn.Parameter((torch.randn(E, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
    w = QuantExpertWeights(w1=G.quantize_tensor(b.w1.detach(), 4, 128), w2=G.quantize_tensor(b.w2.detach(), 4, 128))
    attach_packed_buffers(b, w, torch.bfloat16)
    install_packed_expert_access(b)
    state = {k: v.detach().cpu() for k, v in model.state_dict().items()}
    save_file(state, os.path.join(tmp_path, "model-int4.safetensors"))
    with open(os.path.join(tmp_path, "quantization.json"), "w") as f:
        json.dump({"config": {"bits": 4, "compute_dtype": "bfloat16"},
                   "targets": [{"kind": "expert", "name": "blocks.0"}]}, f)
    return model, state


def test_load_to_device_is_byte_exact(tmp_path):
    from llada_quant_b200 import checkpoint as C
    _, state = _model_and_checkpoint(str(tmp_path))
    path = C.find_weights_file(str(tmp_path))
    got = C.load_to_device(path, "cuda", chunk_bytes=1 << 20)
    ref = load_file(path)
    assert set(got) == set(ref)
    for k in ref:
        assert got[k].is_cuda and got[k].dtype == ref[k].dtype
        assert torch.equal(got[k].cpu(), ref[k])


def test_packed_experts_and_model_restore_compute_the_same_layer(tmp_path):
    from llada_quant_b200 import checkpoint as C
    from llada_quant_b200.fused_moe import moe_layer
    from llada_quant_b200.moe import is_packed_expert_block
    model, _ = _model_and_checkpoint(str(tmp_path))
    x = torch.randn(64, 1024, device="cuda").to(torch.bfloat16)
    ref = moe_layer(x, model.gate, model.blocks.get_submodule("0").packed_experts(), 2)
    blocks = C.load_packed_experts(str(tmp_path), "cuda")
    assert list(blocks) == ["blocks.0"] and blocks["blocks.0"].group_size == 128
    assert torch.equal(moe_layer(x, model.gate, blocks["blocks.0"], 2), ref)
    # a fresh skeleton with BF16 expert parameters absorbs the checkpoint on the GPU
    fresh = torch.nn.Module()
    fb = torch.nn.Module()
    fb.w1 = torch.nn.Parameter(torch.zeros(8, 1024, 1024, dtype=torch.bfloat16, device="cuda"))
    fb.w2 = torch.nn.Parameter(torch.zeros(8, 1024, 512, dtype=torch.bfloat16, device="cuda"))
    fbs = torch.nn.Module()
    fbs.add_module("0", fb)
    fresh.add_module("blocks", fbs)
    fresh.gate = torch.nn.Parameter(torch.zeros(8, 1024, dtype=torch.bfloat16, device="cuda"))
    manifest = C.restore_quantized_weights(fresh, str(tmp_path))
    assert manifest["config"]["bits"] == 4
    blk = fresh.blocks.get_submodule("0")
    assert is_packed_expert_block(blk) and blk._qw1.is_cuda
    assert torch.equal(moe_layer(x, fresh.gate, blk.packed_experts(), 2), ref)
    assert torch.equal(blk.w1, model.blocks.get_submodule("0").w1)  # the PACKED property still dequantizes exactly
