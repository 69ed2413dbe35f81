"""The minimal decode step (paia_gemv.decode): a small model (2 layers, hidden 512, GQA 8/2 heads of 64, qkv bias) in
every format; the token step with the library's GEMVs against the same step with every projection as torch fp32
dequantise-then-matmul of the same bytes: logits within 1e-2 relative L2 (bf16 activations between layers) and the
same argmax token, step after step; the step captured in a CUDA graph gives the same tokens as eager steps."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DIMS = dict(hidden=512, heads=8, kv_heads=2, head_dim=64, inter=1024, vocab=1000, layers=2, qkv_bias=True)


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from paia_gemv import load_lib
    return load_lib()


@pytest.mark.parametrize("kind", ["bf16", "fp8", "int4", "int4_asym"])
def test_decode_step_matches_torch_reference(L, kind):
    from paia_gemv import decode
    m = decode.DecodeModel(L, "qwen25_7b", kind, ctx=32, dims=DIMS, seed=3)
    ref = decode.DecodeModel(L, "qwen25_7b", kind, ctx=32, dims=DIMS, seed=3)   # same seed: same weights, cache
    for t in range(4):
        m.token.fill_(17 + t)
        ref.token.fill_(17 + t)
        a = m.step().float().clone()
        b = ref.step(reference=True).float().clone()
        torch.cuda.synchronize()
        rel = ((a - b).norm() / b.norm()).item()
        assert rel < 1e-2, (kind, t, rel)
        assert int(m.token.item()) == int(ref.token.item()), (kind, t)
    assert L.device_error(1) == 0


def test_decode_step_graph_equals_eager(L):
    from paia_gemv import decode
    m = decode.DecodeModel(L, "llama31_8b", "fp8", ctx=32, dims=dict(DIMS, qkv_bias=False), seed=5)
    m.token.fill_(3)
    eager = []
    for _ in range(3):
        m.step()
        eager.append(int(m.token.item()))
    g_model = decode.DecodeModel(L, "llama31_8b", "fp8", ctx=32, dims=dict(DIMS, qkv_bias=False), seed=5)
    g_model.token.fill_(3)
    g_model.step()                                       # warm-up outside the capture (first-call setup)
    torch.cuda.synchronize()
    g_model.token.fill_(3)                               # every step rewrites the same cache position from its token
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        g_model.step()
    got = []
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        got.append(int(g_model.token.item()))
    assert got == eager
