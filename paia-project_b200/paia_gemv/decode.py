"""A minimal batch-1 decode step built around the GEMV family: the layer structure of Llama-3.1-8B / Qwen2.5-7B with
synthetic weights, every projection through this library's GEMVs, everything else on the device with torch.

One token = embedding -> L x [RMSNorm -> qkv (+ bias) with RoPE fused in its epilogue -> KV-cache write ->
grouped-query attention over the cache -> o -> residual -> RMSNorm -> gate_up -> SiLU(gate) * up -> down -> residual]
-> RMSNorm -> lm_head -> argmax. The cache holds `ctx` positions (the first ctx - 1 synthetic), and the token is decoded
at position ctx - 1, so every tensor shape is fixed and a whole token captures as one CUDA graph; tokens/s = 1 / its
device time. The reference measures decode cost per token as a sum of per-op GEMV times
(paia-bench/bench/analyze_e4.py:177-196); this measures the token itself, GEMVs and the ops between them (torch:
RMSNorm, scaled-dot-product attention, SiLU x up, residual adds).
"""
import torch
import torch.nn.functional as F

from . import quant

MODELS = {
    "llama31_8b": dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336, vocab=128256, layers=32,
                       qkv_bias=False, rope_theta=500000.0),
    "qwen25_7b": dict(hidden=3584, heads=28, kv_heads=4, head_dim=128, inter=18944, vocab=152064, layers=28,
                      qkv_bias=True, rope_theta=1000000.0),
}


class Projection:
    """One weight matrix [N, K] in a format, on the device, with its GEMV through the library (or, for references,
    a torch fp32 dequantise-then-matmul of the same bytes). rope = (rope_rows, head_dim, pos, theta): a fused QKV
    projection whose first rope_rows rows are q / k heads, stored pair-interleaved (quant.rope_pair_rows) and rotated
    in the GEMV's epilogue (paia_gemv_rope); its output is in the natural row order."""

    def __init__(self, lib, kind, N, K, g, bias=False, rope=None):
        self.lib, self.kind, self.N, self.K, self.rope = lib, kind, N, K, rope
        W = torch.randn(N, K, device="cuda", generator=g).mul_(0.02)
        self.s = self.z = None
        if kind == "bf16":
            self.W = W.to(torch.bfloat16)
        elif kind == "fp8":
            self.W, self.s = quant.quantize_fp8_rowwise(W)
        elif kind == "int4":
            self.W, self.s = quant.quantize_int4_g128(W)
        else:
            self.W, self.s, self.z = quant.quantize_int4_asym(W)
        del W
        self.bias = (torch.randn(N, device="cuda", generator=g) * 0.02).to(torch.bfloat16) if bias else None
        self.natural = None
        if rope is not None:
            # row-wise formats: reordering the quantised rows (and their scales / zeros / bias) is reordering W
            rows, hd = rope[0], rope[1]
            perm = lambda t: None if t is None else quant.rope_pair_rows(t, rows, hd)   # noqa: E731
            self.W, self.s, self.z, self.bias = perm(self.W), perm(self.s), perm(self.z), perm(self.bias)
            j = torch.arange(N, device="cuda")
            src = j.clone()
            jh = j[:rows] % hd
            src[:rows] = j[:rows] - jh + (jh >> 1) + (jh & 1) * (hd // 2)
            self.natural = torch.empty_like(src)
            self.natural[src] = j                                    # natural row d sits at stored row natural[d]
        table = {"bf16": lib.variants, "fp8": lib.variants_fp8, "int4": lib.variants_int4,
                 "int4_asym": lib.variants_int4_asym}[kind]
        want = {"bf16": (2, 4, 4, 0, 1), "fp8": (2, 2, 4, 0, 1)}.get(kind, (4, 2, 4, 0, 1))
        self.variant = next(v["id"] for v in table if tuple(v[k] for k in "RUWSH") == want)

    def __call__(self, x, y):
        """y = W x (+ bias) through the library's default path (bf16 in and out), rotated when rope is set."""
        L, p = self.lib, (lambda t: None if t is None else t.data_ptr())
        W, xp, yp, v = self.W.data_ptr(), x.data_ptr(), y.data_ptr(), self.variant
        if self.rope is not None:
            rows, hd, pos, theta = self.rope
            L.rope(self.kind, W, p(self.s), p(self.z), xp, p(self.bias), yp, self.N, self.K, rows, hd, pos, theta)
        elif self.kind == "bf16":
            L.bf16_bias(W, xp, p(self.bias), yp, self.N, self.K, v) if self.bias is not None else \
                L.bf16(W, xp, yp, self.N, self.K, v)
        elif self.kind == "fp8":
            L.fp8_bias(W, p(self.s), xp, p(self.bias), yp, self.N, self.K, v) if self.bias is not None else \
                L.fp8(W, p(self.s), xp, yp, self.N, self.K, v)
        elif self.kind == "int4":
            L.int4_bias(W, p(self.s), xp, p(self.bias), yp, self.N, self.K, v) if self.bias is not None else \
                L.int4(W, p(self.s), xp, yp, self.N, self.K, v)
        else:
            L.int4_asym_bias(W, p(self.s), p(self.z), xp, p(self.bias), yp, self.N, self.K, v) \
                if self.bias is not None else L.int4_asym(W, p(self.s), p(self.z), xp, yp, self.N, self.K, v)
        return y

    def dequantised(self):
        if self.kind == "bf16":
            return self.W.float()
        if self.kind == "fp8":
            return quant.dequant_fp8(self.W, self.s)
        if self.kind == "int4":
            return quant.dequant_int4(self.W, self.s)
        return quant.dequant_int4_asym(self.W, self.s, self.z)

    def reference(self, x, y):
        """The same projection as torch fp32 dequantise-then-matmul (rotated in fp32 when rope is set), rounded to
        bf16 once (for checks)."""
        r = self.dequantised() @ x.float()
        if self.bias is not None:
            r = r + self.bias.float()
        if self.rope is not None:
            rows, hd, pos, theta = self.rope
            r = r[self.natural]
            half = hd // 2
            inv = theta ** (-torch.arange(0, hd, 2, device=r.device, dtype=torch.float64) / hd)
            ang = pos * inv
            cos = torch.cat([ang.cos(), ang.cos()]).float()
            sin = torch.cat([ang.sin(), ang.sin()]).float()
            t = r[:rows].view(-1, hd)
            rot = torch.cat([-t[:, half:], t[:, :half]], dim=1)
            r = torch.cat([(t * cos + rot * sin).reshape(-1), r[rows:]])
        y.copy_(r.to(torch.bfloat16))
        return y

    def weight_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.W, self.s, self.z) if t is not None)


class DecodeModel:
    """Synthetic weights of a model's decode path in one format, a KV cache of `ctx` positions, and the token step.
    `dims` overrides the model's sizes (small models for tests); `layers` limits the layer count."""

    def __init__(self, lib, model, kind, ctx=1024, layers=None, seed=0, dims=None):
        cfg = dict(MODELS[model])
        cfg.update(dims or {})
        if layers is not None:
            cfg["layers"] = layers
        self.cfg, self.kind, self.ctx = cfg, kind, ctx
        H, nh, nkv, hd, I, V = (cfg[k] for k in ("hidden", "heads", "kv_heads", "head_dim", "inter", "vocab"))
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.embed = (torch.randn(V, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        self.layers = []
        # RoPE (rotate-half form) of q and k at the decoded position ctx - 1, in the qkv projection's epilogue
        rope = ((nh + nkv) * hd, hd, float(ctx - 1), float(cfg["rope_theta"]))
        norm = lambda: (1.0 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16).float()   # noqa: E731
        for _ in range(cfg["layers"]):
            self.layers.append({
                "norm1": norm(),
                "norm2": norm(),
                "qkv": Projection(lib, kind, (nh + 2 * nkv) * hd, H, g, bias=cfg["qkv_bias"], rope=rope),
                "o": Projection(lib, kind, H, nh * hd, g),
                "gate_up": Projection(lib, kind, 2 * I, H, g),
                "down": Projection(lib, kind, H, I, g),
                "k": (torch.randn(nkv, ctx, hd, device="cuda", generator=g)).to(torch.bfloat16),
                "v": (torch.randn(nkv, ctx, hd, device="cuda", generator=g)).to(torch.bfloat16),
            })
        self.norm_f = norm()
        self.lm_head = Projection(lib, kind, V, H, g)
        # activations, reused every token (fixed addresses, so the token captures as a CUDA graph)
        dev = dict(device="cuda", dtype=torch.bfloat16)
        self.token = torch.zeros(1, device="cuda", dtype=torch.long)
        self.h = torch.empty(H, **dev)
        self.a = torch.empty(H, **dev)
        self.qkv = torch.empty((nh + 2 * nkv) * hd, **dev)
        self.attn = torch.empty(nh * hd, **dev)
        self.o = torch.empty(H, **dev)
        self.gu = torch.empty(2 * I, **dev)
        self.m = torch.empty(I, **dev)
        self.d = torch.empty(H, **dev)
        self.logits = torch.empty(V, **dev)

    def weight_bytes(self):
        n = self.lm_head.weight_bytes()
        for lay in self.layers:
            n += sum(lay[k].weight_bytes() for k in ("qkv", "o", "gate_up", "down"))
        return n

    @staticmethod
    def _rmsnorm(x, w, out, eps=1e-5):
        """out = bf16(x * rsqrt(mean(x^2) + eps) * w), computed in fp32 (w is kept in fp32)."""
        out.copy_(F.rms_norm(x.float(), (x.numel(),), w, eps))
        return out

    def step(self, reference=False):
        """Decode one token: reads self.token, writes self.logits and the argmax into self.token. reference=True
        runs every projection as torch fp32 dequantise-then-matmul (RoPE in fp32) instead of the library's GEMVs;
        everything else is the same code in both."""
        c = self.cfg
        nh, nkv, hd, I = c["heads"], c["kv_heads"], c["head_dim"], c["inter"]
        proj = (lambda P, x, y: P.reference(x, y)) if reference else (lambda P, x, y: P(x, y))
        self.h.copy_(self.embed.index_select(0, self.token)[0])
        pos = self.ctx - 1
        for lay in self.layers:
            self._rmsnorm(self.h, lay["norm1"], self.a)
            proj(lay["qkv"], self.a, self.qkv)                  # q and k come out rotated
            lay["k"][:, pos].copy_(self.qkv[nh * hd:(nh + nkv) * hd].view(nkv, hd))
            lay["v"][:, pos].copy_(self.qkv[(nh + nkv) * hd:].view(nkv, hd))
            att = F.scaled_dot_product_attention(self.qkv[:nh * hd].view(1, nh, 1, hd), lay["k"].unsqueeze(0),
                                                 lay["v"].unsqueeze(0), enable_gqa=True)
            self.attn.copy_(att.reshape(-1))
            proj(lay["o"], self.attn, self.o)
            self.h.add_(self.o)                                  # bf16 add: fp32 sum rounded once
            self._rmsnorm(self.h, lay["norm2"], self.a)
            proj(lay["gate_up"], self.a, self.gu)
            torch.mul(F.silu(self.gu[:I]), self.gu[I:], out=self.m)
            proj(lay["down"], self.m, self.d)
            self.h.add_(self.d)
        self._rmsnorm(self.h, self.norm_f, self.a)
        proj(self.lm_head, self.a, self.logits)
        self.token.copy_(torch.argmax(self.logits).view(1))
        return self.logits


def time_tokens(model, tokens=20, warmup=3):
    """(device microseconds per token, the token ids decoded): the token step captured as one CUDA graph, replayed
    `tokens` times (each replay decodes the next token from the previous one's argmax)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            model.step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        model.step()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    ids = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(tokens):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ids.append(int(model.token.item()))
    us = e0.elapsed_time(e1) * 1e3 / tokens
    del g
    return us, ids
