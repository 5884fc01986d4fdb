"""HF Qwen3-MoE safetensors checkpoints -> the layouts this library's kernels take.

Reads a checkpoint directory in the hub format (``model.safetensors`` or
shards listed by ``model.safetensors.index.json``; per-expert
``mlp.experts.{e}.{gate,up,down}_proj.weight``, optionally FP8 with
``*_scale_inv`` block scales and ``quantization_config.weight_block_size``)
tensor by tensor, without materialising the whole state dict, and builds for
each layer:

* expert weights in the HF fused layout ``gate_up [E, 2I', H]`` (gate rows,
  then up rows) and ``down [E, H, I']``, ready for ``nkimoe_pack_gate_up /
  nkimoe_pack_down`` with ``NKIMOE_LAYOUT_HF``; ``I' = I + pad`` with zero
  rows/columns when the intermediate size is padded
  (``moe_intermediate_pad_size``, qwen.py:196-201, :213-216);
* FP8 weights dequantised as the reference does (qwen.py:101-116:
  ``fp8.to(f32) * scale_inv`` expanded over the weight blocks, cast to the
  model dtype), on the target device;
* the router in fp32 (the reference's router dtype, qwen.py:261, :276).

The reference's conversion (qwen.py:119-233) writes the NxD layout
``gate_up_proj [E, H, 2I]``; the HF fused layout here is its transpose per
expert, which the pack kernels read directly (no host transpose).
"""

from __future__ import annotations

import json
import os

import torch


class CheckpointReader:
    """Lazy access to the tensors of a (possibly sharded) safetensors checkpoint."""

    def __init__(self, path: str):
        from safetensors import safe_open

        self.dir = path if os.path.isdir(path) else os.path.dirname(path)
        index = os.path.join(self.dir, "model.safetensors.index.json")
        if os.path.isdir(path) and os.path.exists(index):
            weight_map = json.load(open(index))["weight_map"]
            files = sorted(set(weight_map.values()))
        else:
            single = path if not os.path.isdir(path) else os.path.join(path, "model.safetensors")
            files = [os.path.basename(single)]
            weight_map = None
        self._files = {f: safe_open(os.path.join(self.dir, f), framework="pt") for f in files}
        if weight_map is None:
            (f,) = files
            weight_map = {k: f for k in self._files[f].keys()}
        self.weight_map = weight_map
        # hub checkpoints prefix the decoder with "model."; NxD state dicts do not
        self.prefix = "model." if any(k.startswith("model.layers.") for k in weight_map) else ""

    def has(self, name: str) -> bool:
        return name in self.weight_map

    def get(self, name: str) -> torch.Tensor:
        if name not in self.weight_map:
            raise KeyError(f"{name} not in checkpoint {self.dir}")
        return self._files[self.weight_map[name]].get_tensor(name)

    def layer(self, l: int, rest: str) -> str:  # noqa: E741
        return f"{self.prefix}layers.{l}.{rest}"


def dequantize_fp8_blocks(fp8: torch.Tensor, scale_inv: torch.Tensor, block, dtype=torch.bfloat16,
                          device=None) -> torch.Tensor:
    """``fp8 * scale_inv`` with each scale covering a ``block[0] x block[1]``
    tile of the weight (qwen.py:101-116); weights whose sides are not block
    multiples take the leading part of the expanded scales."""
    dev = device if device is not None else fp8.device
    w = fp8.to(dev).to(torch.float32)
    s = scale_inv.to(dev).to(torch.float32)
    s = s.repeat_interleave(block[0], dim=0).repeat_interleave(block[1], dim=1)[: w.shape[0], : w.shape[1]]
    return (w * s).to(dtype)


class Qwen3MoECheckpoint:
    """Per-tensor loader for one checkpoint: weights in the model dtype on
    ``device`` (FP8 dequantised on the way)."""

    def __init__(self, path: str, device="cuda", dtype=torch.bfloat16):
        from transformers import AutoConfig

        self.reader = CheckpointReader(path)
        self.hf_config = AutoConfig.from_pretrained(self.reader.dir)
        self.device = torch.device(device)
        self.dtype = dtype
        q = getattr(self.hf_config, "quantization_config", None) or {}
        if not isinstance(q, dict):
            q = q.to_dict()
        self.block = q.get("weight_block_size")
        self.pad = int(getattr(self.hf_config, "moe_intermediate_pad_size", 0) or 0)

    def tensor(self, name: str, dtype=None) -> torch.Tensor:
        dtype = dtype or self.dtype
        w = self.reader.get(name)
        scale = name + "_scale_inv"
        if self.reader.has(scale):
            if not self.block:
                raise ValueError(f"{scale} present but no quantization_config.weight_block_size")
            return dequantize_fp8_blocks(w, self.reader.get(scale), self.block, dtype, self.device)
        return w.to(self.device, dtype)

    def layer_tensor(self, l: int, rest: str, dtype=None) -> torch.Tensor:  # noqa: E741
        return self.tensor(self.reader.layer(l, rest), dtype)

    def experts(self, l: int):  # noqa: E741
        """Layer ``l``'s experts in the HF fused layout: ``(gate_up [E, 2I', H],
        down [E, H, I'])`` with ``I' = I + pad`` (zero padding)."""
        E = self.hf_config.num_experts
        g0 = self.layer_tensor(l, "mlp.experts.0.gate_proj.weight")
        I, H = g0.shape
        Ip = I + self.pad
        gate_up = torch.zeros(E, 2 * Ip, H, dtype=self.dtype, device=self.device)
        down = torch.zeros(E, H, Ip, dtype=self.dtype, device=self.device)
        for e in range(E):
            gate_up[e, :I] = g0 if e == 0 else self.layer_tensor(l, f"mlp.experts.{e}.gate_proj.weight")
            gate_up[e, Ip:Ip + I] = self.layer_tensor(l, f"mlp.experts.{e}.up_proj.weight")
            down[e, :, :I] = self.layer_tensor(l, f"mlp.experts.{e}.down_proj.weight")
        return gate_up, down
