"""Seeded synthetic operands for the decode GEMV shapes.

There are no checkpoints on the measurement boxes, so every weight matrix, activation vector and bias is synthetic,
with the value distributions of the benchmark configurations: W ~ N(0, 0.02) in fp32 (then bf16 or quantised),
x ~ N(0, 1) in bf16, bias ~ N(0, 0.02) in bf16, drawn in that order from one torch generator seeded with `seed`
(0 by default). On the CPU generator the bytes are identical on every machine running the same torch build, which is
what lets the CPU oracle and the GPU see the same operands. On a CUDA generator the values differ from the CPU ones but
have the same distribution; that is used for the large timing operands.

The reference harness draws uniform values instead (W = (U[0,1) - 0.5) * 0.04, x = U[0,1) - 0.5, seed 1000 + N + K,
paia-bench/bench/ops/ours_bf16.py:70-74); `harness_operands` reproduces that for drop-in comparisons.
"""
import torch

# Llama-3.1-8B and Qwen2.5-7B decode GEMV shapes, [N, K] (paia-bench/configs/shapes.yaml:19-48).
SHAPES = {
    "llama31_8b": {"q_proj": (4096, 4096), "k_proj": (1024, 4096), "v_proj": (1024, 4096), "o_proj": (4096, 4096),
                   "gate_proj": (14336, 4096), "up_proj": (14336, 4096), "down_proj": (4096, 14336),
                   "qkv_fused": (6144, 4096), "gate_up_fused": (28672, 4096), "lm_head": (128256, 4096)},
    "qwen25_7b": {"q_proj": (3584, 3584), "k_proj": (512, 3584), "v_proj": (512, 3584), "o_proj": (3584, 3584),
                  "gate_proj": (18944, 3584), "up_proj": (18944, 3584), "down_proj": (3584, 18944),
                  "qkv_fused": (4608, 3584), "gate_up_fused": (37888, 3584), "lm_head": (152064, 3584)},
}
N_LAYERS = {"llama31_8b": 32, "qwen25_7b": 28}
# The fused per-layer GEMV sequence of one decode step, in execution order.
LAYER_SEQUENCE = ("qkv_fused", "o_proj", "gate_up_fused", "down_proj")


def generator(seed=0, device="cpu"):
    return torch.Generator(device=device).manual_seed(seed)


def weights_f32(N, K, g, device="cpu"):
    """W ~ N(0, 1) * 0.02, float32 [N, K]."""
    return torch.randn(N, K, generator=g, device=device, dtype=torch.float32).mul_(0.02)


def activation_bf16(K, g, device="cpu"):
    """x ~ N(0, 1), bf16 [K]."""
    return torch.randn(K, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


def bias_bf16(N, g, device="cpu"):
    """bias ~ N(0, 1) * 0.02, bf16 [N]."""
    return torch.randn(N, generator=g, device=device, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)


def operands(N, K, seed=0, device="cpu", with_bias=False):
    """(W fp32 [N,K], x bf16 [K], bias bf16 [N] or None), drawn in that order from one generator."""
    g = generator(seed, device)
    W = weights_f32(N, K, g, device)
    x = activation_bf16(K, g, device)
    b = bias_bf16(N, g, device) if with_bias else None
    return W, x, b


def harness_operands(N, K, M=1, device="cuda"):
    """The reference harness's operands: W = (U - 0.5) * 0.04 fp32, x = (U - 0.5) bf16 [M, K], seed 1000 + N + K
    (paia-bench/bench/ops/ours_bf16.py:70-74, ours_quant.py:63-66)."""
    g = torch.Generator(device=device).manual_seed(1000 + N + K)
    W = (torch.rand(N, K, device=device, generator=g, dtype=torch.float32) - 0.5).mul_(0.04)
    x = (torch.rand(M, K, device=device, generator=g) - 0.5).to(torch.bfloat16)
    return W, x
