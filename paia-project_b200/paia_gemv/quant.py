"""Torch quantisers and dequantisers for the weight formats (CPU or CUDA tensors).

The formats are the reference's, byte for byte (Bejaine/PAIA-Project src/paia_gemv/quant.py:1-38 and
quant_host.h:1-13), plus the asymmetric INT4 convention of paia-bench/bench/ops/lib_quant.py:159-167:

  FP8 W8A16   per output row: scale = amax / 448 (1 for an all-zero row), q = e4m3fn(w / scale) with round-to-nearest-
              even and saturation at 448; codes 0x7F / 0xFF (NaN) are never produced.
  INT4 sym    per group of 128 along K: s = fp16(amax / 7) (1 when amax == 0; a zero fp16 scale divides as 1),
              n = clamp(rint(w / s), -7, 7) + 8 in 1..15; w ~ (n - 8) * s.
  INT4 asym   per group of 128 along K: scale = max(max - min, 1e-6) / 15, q = clamp(rint((w - min) / scale), 0, 15),
              zero = min + 8 * scale (fp32), stored as bf16 scale and bf16 zero; w ~ (q - 8) * scale + zero.
  packing     both INT4 formats: uint8 [N, K/2], byte j = q[2j] | q[2j+1] << 4 (even k in the low nibble).
"""
import torch

GROUP = 128


def pack_nibbles(q):
    """int tensor [N, K] of values 0..15 -> uint8 [N, K/2] (even k in the low nibble)."""
    q = q.to(torch.int32)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).to(torch.uint8).contiguous()


def unpack_nibbles(packed):
    """uint8 [N, K/2] -> int32 [N, K] values 0..15."""
    p = packed.to(torch.int32)
    return torch.stack([p & 0xF, p >> 4], dim=-1).reshape(p.shape[0], p.shape[1] * 2)


def quantize_fp8_rowwise(W):
    """W float32 [N, K] -> (q uint8 [N, K] e4m3fn codes, scale float32 [N])."""
    W = W.float()
    amax = W.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    codes = torch.clamp(W / scale[:, None], -448.0, 448.0).to(torch.float8_e4m3fn)
    return codes.view(torch.uint8).contiguous(), scale.contiguous()


def dequant_fp8(q, scale):
    return q.view(torch.float8_e4m3fn).float() * scale.float()[:, None]


def quantize_int4_g128(W):
    """W float32 [N, K], K % 128 == 0 -> (packed uint8 [N, K/2], scales float16 [N, K/128])."""
    W = W.float()
    N, K = W.shape
    if K % GROUP:
        raise ValueError("K % 128 required")
    g = W.reshape(N, K // GROUP, GROUP)
    amax = g.abs().amax(dim=-1)
    s16 = torch.where(amax > 0, amax / 7.0, torch.ones_like(amax)).to(torch.float16)
    div = s16.float()
    div = torch.where(div > 0, div, torch.ones_like(div))
    n = torch.clamp(torch.round(g / div[..., None]), -7, 7) + 8
    return pack_nibbles(n.reshape(N, K)), s16.contiguous()


def dequant_int4(packed, s16):
    n = unpack_nibbles(packed).float() - 8.0
    return n * s16.float().repeat_interleave(GROUP, dim=1)


def quantize_int4_asym(W):
    """W float32 [N, K], K % 128 == 0 -> (packed uint8 [N, K/2], scale bf16 [N, K/128], zero bf16 [N, K/128])."""
    W = W.float()
    N, K = W.shape
    if K % GROUP:
        raise ValueError("K % 128 required")
    g = W.reshape(N, K // GROUP, GROUP)
    lo, hi = g.amin(dim=-1), g.amax(dim=-1)
    scale = torch.clamp(hi - lo, min=1e-6) / 15.0
    q = torch.clamp(torch.round((g - lo[..., None]) / scale[..., None]), 0, 15)
    zero = lo + 8 * scale
    return pack_nibbles(q.reshape(N, K)), scale.to(torch.bfloat16).contiguous(), zero.to(torch.bfloat16).contiguous()


def dequant_int4_asym(packed, scale_bf16, zero_bf16):
    n = unpack_nibbles(packed).float() - 8.0
    s = scale_bf16.float().repeat_interleave(GROUP, dim=1)
    z = zero_bf16.float().repeat_interleave(GROUP, dim=1)
    return n * s + z


def rope_pair_rows(t, rope_rows, head_dim):
    """Rows of a fused QKV projection (weights, scales, zeros or bias; any format, rows first) reordered for the
    rotary epilogue (paia_gemv_rope): within each of the rope_rows // head_dim q/k heads, new row 2i + h holds old row
    i + h head_dim / 2 (the two halves a rotate-half RoPE pairs become adjacent); rows past rope_rows stay."""
    import torch as _torch
    half = head_dim // 2
    j = _torch.arange(rope_rows, device=t.device)
    base = j - j % head_dim
    jh = j % head_dim
    src = base + (jh >> 1) + (jh & 1) * half
    out = t.clone()
    out[:rope_rows] = t[src]
    return out

