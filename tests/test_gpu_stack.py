"""Decoder stack on this library's kernels against HF ``Qwen3MoeForCausalLM``.

The reference validates a model by greedy generation with teacher forcing at
divergence, comparing logits per position (``main.py:296-378``; tolerances
``main.py:555``).  Here the HF model runs in fp32 on the CPU with bf16-valued
weights (fp32 router), the stack in bf16 on the GPU, and the check is per
position: cosine of the logit vectors, the normwise error
max|l - l_ref| / max|l_ref|, and agreement of the argmax token.  Bars (bf16
activations through the layers): at >= 95% of positions cosine >= 0.999 and
normwise <= 0.05 (the reference's rtol for all logits); every position cosine
>= 0.95; argmax agreement >= 0.9.  The allowance covers positions where the
bf16 rounding of an activation moves a near-tied top-k expert choice in some
layer (about 2 in 100 tokens here), which the reference's teacher-forced
check also absorbs.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

COS_BAR = 0.999
NORM_BAR = 0.05
QUANTILE = 0.95
COS_FLOOR = 0.95
ARGMAX_BAR = 0.9


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def tiny_hf(seed=0):
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    cfg = Qwen3MoeConfig(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=128, moe_intermediate_size=128,
                         num_experts=8, num_experts_per_tok=2, norm_topk_prob=True,
                         rope_parameters={"rope_type": "default", "rope_theta": 1e6}, rms_norm_eps=1e-6,
                         max_position_embeddings=512, tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    m = Qwen3MoeForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "norm" in name:
                v = 1 + 0.1 * torch.randn_like(p)
            elif name.endswith("mlp.gate.weight"):
                # fp32 router, used unrounded; wide logit gaps, so that the bf16
                # rounding of the activations rarely moves a top-2 choice
                p.copy_(torch.randn_like(p) * 0.5)
                continue
            else:
                v = torch.randn_like(p) * 0.05
            p.copy_(v.bfloat16().float())
    return m


def _check(ours, ref):
    """Per-position cosine / normwise error / argmax over [N, V] against the bars."""
    o, r = ours.float().cpu(), ref.float().cpu()
    cos = torch.nn.functional.cosine_similarity(o, r, dim=-1)
    norm = (o - r).abs().amax(-1) / r.abs().amax(-1)
    good = ((cos >= COS_BAR) & (norm <= NORM_BAR)).float().mean().item()
    agree = (o.argmax(-1) == r.argmax(-1)).float().mean().item()
    msg = f"good {good:.3f}, min cos {cos.min():.4f} (pos {int(cos.argmin())}), argmax {agree:.3f}"
    assert good >= QUANTILE and cos.min().item() >= COS_FLOOR and agree >= ARGMAX_BAR, msg


@pytest.fixture(scope="module")
def pair():
    from nki_moe_b200.qwen_stack import Qwen3MoEStack

    hf = tiny_hf()
    return hf, Qwen3MoEStack.from_hf(hf, max_batch=4, max_seq=128)


def test_prefill_logits_match_hf(pair):
    hf, st = pair
    ids = torch.randint(0, 1024, (3, 40), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = hf(ids).logits
    ours = st.prefill(ids, all_logits=True)
    _check(ours.reshape(-1, 1024), ref.reshape(-1, 1024))


@pytest.mark.parametrize("graph", [False, True])
def test_decode_teacher_forced_matches_hf(pair, graph):
    """KV-cache decode steps fed the HF greedy tokens (teacher forcing)."""
    hf, st = pair
    prompt = torch.randint(0, 1024, (2, 17), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        gen = hf.generate(prompt, max_new_tokens=8, do_sample=False, return_dict_in_generate=True,
                          output_scores=True, attention_mask=torch.ones_like(prompt))
    ref_scores = torch.stack(gen.scores, 1)  # [B, 8, V]
    ref_tokens = gen.sequences[:, prompt.shape[1]:]
    logits = [st.prefill(prompt)]
    for i in range(7):
        logits.append(st.decode(ref_tokens[:, i].cuda(), graph=graph))
    ours = torch.stack(logits, 1)
    _check(ours.reshape(-1, 1024), ref_scores.reshape(-1, 1024))
    st.release_graph()


def test_graph_decode_equals_eager(pair):
    _, st = pair
    prompt = torch.randint(0, 1024, (2, 9), generator=torch.Generator().manual_seed(3))
    toks = torch.randint(0, 1024, (2, 5), generator=torch.Generator().manual_seed(4)).cuda()
    outs = []
    for graph in (False, True):
        st.prefill(prompt)
        outs.append(torch.stack([st.decode(toks[:, i], graph=graph) for i in range(5)], 1).clone())
    st.release_graph()
    assert torch.equal(outs[0], outs[1])


def test_generate_timing_keys(pair):
    _, st = pair
    prompt = torch.randint(0, 1024, (2, 12), generator=torch.Generator().manual_seed(5))
    toks, t = st.generate(prompt, 6)
    st.release_graph()
    assert toks.shape == (2, 6)
    assert t["ttft_ms"] > 0 and t["decode_tok_s"] > 0 and t["decode_steps"] == 5


@pytest.mark.parametrize("fp8", [False, True])
def test_from_safetensors_equals_from_hf(tmp_path, fp8):
    """A hub-format checkpoint (per-expert weights; FP8 blocks with inverse
    scales) loaded tensor by tensor gives the same stack as the in-memory HF
    model holding the same (dequantised) weights: identical logits."""
    import copy
    import json

    from safetensors.torch import load_file, save_file

    from nki_moe_b200.qwen_stack import Qwen3MoEStack
    from oracle import hf_convert

    hf = tiny_hf(seed=7)
    hf.save_pretrained(tmp_path, safe_serialization=True)
    if fp8:
        sd = load_file(str(tmp_path / "model.safetensors"))
        ref_model = copy.deepcopy(hf)
        params = dict(ref_model.named_parameters())
        for k in [k for k in sd if ".mlp.experts." in k]:
            w = sd[k].float()
            scale = torch.zeros(w.shape[0] // 128, w.shape[1] // 128)
            q = torch.empty_like(w, dtype=torch.float8_e4m3fn)
            for i in range(scale.shape[0]):
                for j in range(scale.shape[1]):
                    t = w[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128]
                    scale[i, j] = t.abs().max().clamp(min=1e-8) / 448.0
                    q[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128] = (t / scale[i, j]).to(torch.float8_e4m3fn)
            sd[k], sd[k + "_scale_inv"] = q, scale
        save_file(sd, str(tmp_path / "model.safetensors"))
        cfg = json.load(open(tmp_path / "config.json"))
        cfg["quantization_config"] = {"quant_method": "fp8", "weight_block_size": [128, 128]}
        json.dump(cfg, open(tmp_path / "config.json", "w"))
        # the reference model holds the dequantised expert weights (qwen.py:101-116)
        with torch.no_grad():
            for li, lyr in enumerate(ref_model.model.layers):
                ex = lyr.mlp.experts
                for e in range(ex.gate_up_proj.shape[0]):
                    deq = {n: hf_convert.dequantize_fp8_blocks(sd[f"model.layers.{li}.mlp.experts.{e}.{n}.weight"],
                                                               sd[f"model.layers.{li}.mlp.experts.{e}.{n}.weight_scale_inv"],
                                                               (128, 128), torch.float32)
                           for n in ("gate_proj", "up_proj", "down_proj")}
                    I = deq["gate_proj"].shape[0]
                    ex.gate_up_proj[e, :I] = deq["gate_proj"]
                    ex.gate_up_proj[e, I:] = deq["up_proj"]
                    ex.down_proj[e] = deq["down_proj"]
        hf = ref_model
    a = Qwen3MoEStack.from_hf(hf, max_batch=2, max_seq=64)
    b = Qwen3MoEStack.from_safetensors(str(tmp_path), max_batch=2, max_seq=64)
    ids = torch.randint(0, 1024, (2, 24), generator=torch.Generator().manual_seed(9))
    assert torch.equal(a.prefill(ids, all_logits=True), b.prefill(ids, all_logits=True))


def _ep_stack_worker(rank, world, port, out_dir, overlap=-1):
    """One rank of an expert-parallel decoder stack (each rank: its own two
    sequences, E / P experts) next to a single-GPU stack with the same seed on
    the same GPU (all experts)."""
    import datetime
    import os

    import numpy as np
    import torch.distributed as dist

    from nki_moe_b200.qwen_stack import Qwen3MoEConfig, Qwen3MoEStack
    from nki_moe_b200 import _lib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    _lib.set_option("ep_overlap", overlap)
    cfg = Qwen3MoEConfig(vocab_size=1024, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                         num_key_value_heads=2, head_dim=128, moe_intermediate_size=128, num_experts=8,
                         num_experts_per_tok=2)
    ids = torch.randint(0, 1024, (2 * world, 20), generator=torch.Generator().manual_seed(11))[2 * rank:2 * rank + 2]
    toks = torch.randint(0, 1024, (2, 4), generator=torch.Generator().manual_seed(12 + rank)).cuda()
    ep = Qwen3MoEStack.random_init(cfg, seed=5, max_batch=2, max_seq=64, std=0.05, expert_parallel=True)
    one = Qwen3MoEStack.random_init(cfg, seed=5, max_batch=2, max_seq=64, std=0.05)
    res = {}
    for name, st in (("ep", ep), ("one", one)):
        res[f"{name}_prefill"] = st.prefill(ids, all_logits=True).float().cpu()
        for graph in (False, True):
            st.prefill(ids)
            res[f"{name}_decode_{graph}"] = torch.stack([st.decode(toks[:, i], graph=graph)
                                                        for i in range(4)], 1).float().cpu()
        st.release_graph()
    torch.cuda.synchronize()
    ep.close()
    for k, v in res.items():
        np.save(os.path.join(out_dir, f"{k}_{rank}.npy"), v.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("overlap", [-1, 2])
def test_expert_parallel_stack_two_gpus(tmp_path, overlap):
    """Expert-parallel decoder stack on 2 GPUs (peer-memory exchange in every
    layer, decode step captured in one CUDA graph with device-side epochs)
    against the single-GPU stack of the same weights: logits within the bars
    above (the exchange rounds each rank's partial sum to bf16), graph decode
    bit-identical to eager decode.  With the default schedule (one block at
    these sizes) and with the copy-engine schedule forced, whose side-stream
    copies are then captured into the decode graph."""
    import socket

    import numpy as np
    import torch.multiprocessing as mp
    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    world = 2
    mp.start_processes(_ep_stack_worker, args=(world, port, str(tmp_path), overlap), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        ld = lambda k: torch.from_numpy(np.load(tmp_path / f"{k}_{r}.npy"))  # noqa: E731
        _check(ld("ep_prefill").reshape(-1, 1024), ld("one_prefill").reshape(-1, 1024))
        _check(ld("ep_decode_False").reshape(-1, 1024), ld("one_decode_False").reshape(-1, 1024))
        assert torch.equal(ld("ep_decode_True"), ld("ep_decode_False"))
