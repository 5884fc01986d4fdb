"""Test infrastructure only: CPU restatement of the reference's HF -> NxD
checkpoint conversion for the MoE layers, used as the oracle of the
safetensors loader.  Not a product path.

* FP8 block dequantisation, ``qwen.py:101-116`` (``maybe_dequantize_layer``):
  ``w = fp8.to(f32) * scale_inv.repeat_interleave(b0, 0).repeat_interleave(b1, 1)``,
  then cast to the model dtype.
* Expert layout, ``qwen.py:164-219`` (``convert_qwen3_moe_hf_to_neuron_state_dict``):
  per expert ``gate_proj.weight [I, H]`` and ``up_proj.weight [I, H]`` transposed
  into ``gate_up_proj [E, H, 2I]`` (gate columns first), ``down_proj.weight
  [H, I]`` transposed into ``down_proj [E, I, H]``; with
  ``moe_intermediate_pad_size`` p, gate_up is viewed ``[E, H, 2, I]`` and padded
  right by p, down padded by p rows (``:196-201``, ``:213-216``).
"""

from __future__ import annotations

import torch


def dequantize_fp8_blocks(fp8: torch.Tensor, scale_inv: torch.Tensor, block, dtype=torch.bfloat16):
    """``qwen.py:101-116``."""
    scales = scale_inv.repeat_interleave(block[0], dim=0).repeat_interleave(block[1], dim=1)
    return (fp8.to(torch.float32) * scales.to(torch.float32)).to(dtype)


def experts_to_nxd(gate, up, down, pad: int = 0):
    """``qwen.py:164-219``: lists of per-expert ``gate/up [I, H]`` and ``down
    [H, I]`` -> (``gate_up_proj [E, H, 2(I+p)]``, ``down_proj [E, I+p, H]``)."""
    E = len(gate)
    I, H = gate[0].shape
    gate_up = torch.empty(E, H, 2 * I, dtype=gate[0].dtype)
    for e in range(E):
        gate_up[e, :, :I] = gate[e].T
        gate_up[e, :, I:] = up[e].T
    if pad > 0:
        gate_up = torch.nn.functional.pad(gate_up.reshape(E, H, 2, I), (0, pad)).reshape(E, H, -1)
    dn = torch.empty(E, I, H, dtype=down[0].dtype)
    for e in range(E):
        dn[e] = down[e].T
    if pad > 0:
        dn = torch.nn.functional.pad(dn, (0, 0, 0, pad))
    return gate_up, dn
