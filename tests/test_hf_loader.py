"""The safetensors loader's host side against the reference's conversion
(qwen.py:101-226, restated in ``oracle/hf_convert.py``): FP8 block
dequantisation, per-expert -> stacked expert layouts, intermediate padding,
sharded checkpoints.  CPU only."""

import json

import pytest
import torch

from nki_moe_b200.hf_loader import CheckpointReader, Qwen3MoECheckpoint, dequantize_fp8_blocks
from oracle import hf_convert

E, H, I, LAYERS = 4, 256, 128, 2


def _quantize(w: torch.Tensor, block=(128, 128)):
    """Per-block FP8 (e4m3) quantisation with inverse scales, as FP8 hub checkpoints store them."""
    r, c = w.shape
    sb = torch.zeros((r + block[0] - 1) // block[0], (c + block[1] - 1) // block[1])
    q = torch.empty(r, c, dtype=torch.float8_e4m3fn)
    for i in range(sb.shape[0]):
        for j in range(sb.shape[1]):
            t = w[i * block[0]:(i + 1) * block[0], j * block[1]:(j + 1) * block[1]].float()
            s = t.abs().max().clamp(min=1e-8) / 448.0
            sb[i, j] = s
            q[i * block[0]:(i + 1) * block[0], j * block[1]:(j + 1) * block[1]] = (t / s).to(torch.float8_e4m3fn)
    return q, sb


def _write_checkpoint(d, fp8=False, pad=0, shards=1, seed=0):
    from safetensors.torch import save_file
    from transformers import Qwen3MoeConfig

    g = torch.Generator().manual_seed(seed)
    cfg = Qwen3MoeConfig(vocab_size=64, hidden_size=H, intermediate_size=512, num_hidden_layers=LAYERS,
                         num_attention_heads=2, num_key_value_heads=1, head_dim=128, moe_intermediate_size=I,
                         num_experts=E, num_experts_per_tok=2, norm_topk_prob=True, tie_word_embeddings=False)
    cfg.save_pretrained(d)
    raw = json.load(open(d / "config.json"))
    if fp8:
        raw["quantization_config"] = {"quant_method": "fp8", "weight_block_size": [128, 128]}
    if pad:
        raw["moe_intermediate_pad_size"] = pad
    json.dump(raw, open(d / "config.json", "w"))
    tensors, ref = {}, {}
    for l in range(LAYERS):  # noqa: E741
        gs, us, ds = [], [], []
        for e in range(E):
            for name, shape, lst in (("gate_proj", (I, H), gs), ("up_proj", (I, H), us), ("down_proj", (H, I), ds)):
                w = (torch.randn(*shape, generator=g) * 0.05).to(torch.bfloat16)
                key = f"model.layers.{l}.mlp.experts.{e}.{name}.weight"
                if fp8:
                    q, s = _quantize(w)
                    tensors[key], tensors[key + "_scale_inv"] = q, s
                    lst.append(hf_convert.dequantize_fp8_blocks(q, s, (128, 128)))
                else:
                    tensors[key] = w
                    lst.append(w)
        ref[l] = hf_convert.experts_to_nxd(gs, us, ds, pad)
    keys = sorted(tensors)
    if shards == 1:
        save_file(tensors, str(d / "model.safetensors"))
    else:
        wm = {}
        for i in range(shards):
            part = {k: tensors[k] for k in keys[i::shards]}
            fname = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
            save_file(part, str(d / fname))
            wm.update({k: fname for k in part})
        json.dump({"metadata": {}, "weight_map": wm}, open(d / "model.safetensors.index.json", "w"))
    return ref


def test_fp8_dequantisation_matches_reference():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(256, 384, generator=g) * 0.1
    q, s = _quantize(w)
    ours = dequantize_fp8_blocks(q, s, (128, 128), torch.bfloat16)
    ref = hf_convert.dequantize_fp8_blocks(q, s, (128, 128), torch.bfloat16)
    assert torch.equal(ours, ref)
    assert (ours.float() - w).abs().max() < 0.02  # e4m3 with per-block scales


def test_fp8_dequantisation_ragged_blocks():
    """Weights whose sides are not block multiples use the leading scales."""
    g = torch.Generator().manual_seed(2)
    w = torch.randn(200, 300, generator=g)
    q, s = _quantize(w)
    ours = dequantize_fp8_blocks(q, s, (128, 128), torch.float32)
    for i in range(200):
        for j in (0, 127, 128, 299):
            assert ours[i, j] == q[i, j].float() * s[i // 128, j // 128]


@pytest.mark.parametrize("fp8,pad", [(False, 0), (True, 0), (False, 64), (True, 64)])
def test_experts_match_reference_layout(tmp_path, fp8, pad):
    ref = _write_checkpoint(tmp_path, fp8=fp8, pad=pad)
    ck = Qwen3MoECheckpoint(str(tmp_path), device="cpu")
    assert ck.pad == pad
    for l in range(LAYERS):  # noqa: E741
        gate_up, down = ck.experts(l)
        ref_gu, ref_dn = ref[l]  # NxD layout [E, H, 2I'], [E, I', H]
        assert gate_up.shape == (E, 2 * (I + pad), H) and down.shape == (E, H, I + pad)
        assert torch.equal(gate_up.transpose(1, 2), ref_gu)
        assert torch.equal(down.transpose(1, 2), ref_dn)


def test_sharded_checkpoint(tmp_path):
    ref = _write_checkpoint(tmp_path, shards=3)
    r = CheckpointReader(str(tmp_path))
    assert len(r._files) == 3 and r.prefix == "model."
    gate_up, _ = Qwen3MoECheckpoint(str(tmp_path), device="cpu").experts(1)
    assert torch.equal(gate_up.transpose(1, 2), ref[1][0])
