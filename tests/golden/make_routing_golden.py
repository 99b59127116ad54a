"""Generates tests/golden/routing.npz: routing and FP8 golden vectors from published implementations.

Run in a container where Hugging Face `transformers` is importable (this fixture was made with
transformers 5.5.0 on torch 2.11.0, CPU):

    python tests/golden/make_routing_golden.py

The reference runs its router inside its mistral.rs fork, which is not in its tree, so its routing
has no output to compare against. These fixtures pin the oracle to code it shares nothing with:

  * qwen_*  Hugging Face `Qwen3MoeTopKRouter.forward` (modeling_qwen3_moe.py): softmax over all
            experts in f32, torch.topk, and with norm_topk_prob the division by the k weights' sum.
            The module runs in f32 on bf16-valued inputs: the reference's own router copy holds the
            gate as f32 and takes f32 logits (provider.rs:618-629, cached_layer.rs:1241-1242).
            c1 = config 1 (E16 k2 H1024), both with and without renormalisation; c2 = config 2
            (E128 k8 H2048, renormalised); ties = E128 k8 logits on a 1/8 grid, so many exact ties.
  * dsv3_*  Hugging Face `DeepseekV3TopkRouter.forward` + `DeepseekV3MoE.route_tokens_to_experts`
            (modeling_deepseek_v3.py): sigmoid scores, e_score_correction_bias for the choice,
            group score = sum of the group's top-2, topk_group groups, top-k in them, weights =
            unbiased scores / (sum + 1e-20) * routed_scaling_factor. Config 5's routing (E256 k8,
            8 groups, top-4 groups, scale 2.5) on H = 512 (the selection does not depend on H; the
            full 7168-wide gate would make the fixture 4 MB). c5 = random logits, ties = logits on
            a 1/8 grid. The bias is small enough that every biased score stays positive, where
            HF's masked_fill(0.0) and the -inf mask of DeepSeek-V3's own inference code agree.
  * fp8_*   torch's float8_e4m3fn decode of all 256 codes, and Hugging Face
            `finegrained_fp8.Fp8Dequantize.convert` (the 128x128 block dequantisation of
            DeepSeek-V3 checkpoints: weight.to(f32) * weight_scale_inv per block) on a 256x256
            matrix holding every non-NaN code, with four block scales.

Logit-level fixtures put the router's weight as the identity (hidden size = E), so F.linear passes
the given logits through unchanged (x * 1 + 0 is exact in f32).

The tests never import transformers; they only read the committed .npz.
"""
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

import transformers  # noqa: E402
from transformers.integrations.finegrained_fp8 import Fp8Dequantize  # noqa: E402
from transformers.models.deepseek_v3 import modeling_deepseek_v3 as dsv3  # noqa: E402
from transformers.models.qwen3_moe import modeling_qwen3_moe as qwen  # noqa: E402

from oracle import oracle as O  # noqa: E402  (bf16 rounding of the inputs only)


def bf16_pair(rng, shape, std):
    """Seeded N(0, std) values rounded to bf16: (uint16 bits, their exact f32 values)."""
    bits = O.f32_to_bf16((rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32))
    return bits, O.bf16_to_f32(bits).reshape(shape)


def qwen_route(x32: np.ndarray, w32: np.ndarray, k: int, renorm: bool):
    E, H = w32.shape
    cfg = types.SimpleNamespace(num_experts_per_tok=k, num_experts=E, norm_topk_prob=renorm, hidden_size=H)
    router = qwen.Qwen3MoeTopKRouter(cfg).float()
    with torch.no_grad():
        router.weight.copy_(torch.from_numpy(w32))
        h = torch.from_numpy(x32)
        logits = torch.nn.functional.linear(h, router.weight)
        _, weights, ids = router(h)
    return logits.numpy(), ids.numpy().astype(np.int32), weights.numpy().astype(np.float32)


def dsv3_route(x32: np.ndarray, w32: np.ndarray, bias: np.ndarray, k: int, n_group: int, topk_group: int,
               scale: float):
    E, H = w32.shape
    cfg = types.SimpleNamespace(
        n_routed_experts=E, hidden_size=H, num_local_experts=E, moe_intermediate_size=8, hidden_act="silu",
        n_group=n_group, topk_group=topk_group, norm_topk_prob=True, routed_scaling_factor=scale,
        num_experts_per_tok=k, n_shared_experts=1, intermediate_size=8, pretraining_tp=1, mlp_bias=False)
    moe = dsv3.DeepseekV3MoE(cfg).float()
    with torch.no_grad():
        moe.gate.weight.copy_(torch.from_numpy(w32))
        moe.gate.e_score_correction_bias.copy_(torch.from_numpy(bias))
        logits = moe.gate(torch.from_numpy(x32))
        ids, weights = moe.route_tokens_to_experts(logits)
    return logits.numpy(), ids.numpy().astype(np.int32), weights.numpy().astype(np.float32)


def main():
    rng = np.random.Generator(np.random.Philox(20261202))
    out = {}

    # Qwen3-MoE, config 1 (E16 k2 H1024) with and without renormalisation, and config 2
    xb, x32 = bf16_pair(rng, (64, 1024), 1.0)
    wb, w32 = bf16_pair(rng, (16, 1024), 0.02)
    out["qwen_c1_x"], out["qwen_c1_w"] = xb, wb
    lg, ids, w = qwen_route(x32, w32, 2, True)
    out["qwen_c1_logits"], out["qwen_c1_renorm_ids"], out["qwen_c1_renorm_weights"] = lg, ids, w
    _, ids, w = qwen_route(x32, w32, 2, False)
    out["qwen_c1_plain_ids"], out["qwen_c1_plain_weights"] = ids, w

    xb, x32 = bf16_pair(rng, (48, 2048), 1.0)
    wb, w32 = bf16_pair(rng, (128, 2048), 0.02)
    out["qwen_c2_x"], out["qwen_c2_w"] = xb, wb
    lg, ids, w = qwen_route(x32, w32, 8, True)
    out["qwen_c2_logits"], out["qwen_c2_ids"], out["qwen_c2_weights"] = lg, ids, w

    # ties: logits on a 1/8 grid, passed through an identity gate
    tl = (np.round(rng.standard_normal((64, 128), dtype=np.float32) * 8.0) / 8.0).astype(np.float32)
    _, ids, w = qwen_route(tl, np.eye(128, dtype=np.float32), 8, True)
    out["qwen_ties_logits"], out["qwen_ties_ids"], out["qwen_ties_weights"] = tl, ids, w

    # DeepSeek-V3 group-limited routing, config 5's selection (E256 k8, 8 groups, top-4, x2.5)
    xb, x32 = bf16_pair(rng, (64, 512), 1.0)
    wb, w32 = bf16_pair(rng, (256, 512), 0.02)
    bias = (rng.uniform(-0.05, 0.05, 256)).astype(np.float32)
    out["dsv3_c5_x"], out["dsv3_c5_w"], out["dsv3_bias"] = xb, wb, bias
    lg, ids, w = dsv3_route(x32, w32, bias, 8, 8, 4, 2.5)
    out["dsv3_c5_logits"], out["dsv3_c5_ids"], out["dsv3_c5_weights"] = lg, ids, w
    tl = (np.round(rng.standard_normal((64, 256), dtype=np.float32) * 4.0) / 8.0).astype(np.float32)
    _, ids, w = dsv3_route(tl, np.eye(256, dtype=np.float32), bias, 8, 8, 4, 2.5)
    out["dsv3_ties_logits"], out["dsv3_ties_ids"], out["dsv3_ties_weights"] = tl, ids, w

    # FP8 e4m3fn: every code's value, and the 128x128 block dequantisation of DeepSeek-V3 weights
    codes = np.arange(256, dtype=np.uint8)
    out["fp8_code_values"] = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    finite = codes[(codes & 0x7F) != 0x7F]
    q = rng.choice(finite, size=(256, 256)).astype(np.uint8)
    q[0, :finite.size] = finite  # every finite code appears at least once
    s = np.array([[0.5, 3.0e-4], [1.7e-3, 2.0 ** -12]], dtype=np.float32)
    quantizer = types.SimpleNamespace(quantization_config=types.SimpleNamespace(weight_block_size=(128, 128)))
    deq = Fp8Dequantize(quantizer).convert({"weight$": [torch.from_numpy(q).view(torch.float8_e4m3fn)],
                                            "weight_scale_inv": [torch.from_numpy(s)]}, full_layer_name="w")["w"]
    out["fp8_q"], out["fp8_scales"], out["fp8_dequant"] = q, s, deq.numpy().astype(np.float32)

    out["versions"] = np.array([f"transformers {transformers.__version__}", f"torch {torch.__version__}"])
    np.savez_compressed(os.path.join(HERE, "routing.npz"), **out)
    print("wrote routing.npz:", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
