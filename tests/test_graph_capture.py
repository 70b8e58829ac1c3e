"""The kernels of one op run back to back on one stream, and several are launched with
programmatic stream serialization: the pair-bias token projection beside the z-bias
kernel, the dead-row vote beside the attention, the gate's set-up before the previous
kernel ends. These tests replay each op from a CUDA graph (where those launches become
programmatic graph edges) twice over and require the result to equal the eager call's
bit for bit, with a masked key tail so that the dead-row kernel takes part."""
import pytest
import torch

from helpers import rnd
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu


def _replay_equals_eager(fn):
    eager = fn().clone()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        out = fn()
    for _ in range(2):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)


def test_attn_pair_bias_graph_replay(device):
    M, C, H, D = 384, 128, 4, 32
    X = rnd(M, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=1)
    Z = rnd(M, M, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=2)
    WQ, WK, WV, Wg, Wo = (rnd(C, C, dtype=torch.bfloat16, device=device, sd=C**-0.5, seed=s) for s in range(3, 8))
    W_ln = 1.0 + rnd(C, dtype=torch.bfloat16, device=device, sd=0.1, seed=9)
    B_ln = rnd(C, dtype=torch.bfloat16, device=device, sd=0.1, seed=10)
    W_pz = rnd(C, H, dtype=torch.bfloat16, device=device, sd=C**-0.5, seed=11)
    km = torch.ones(M, dtype=torch.bool, device=device)
    km[-40:] = False
    pre = tops.attn_pair_bias.precompute(WQ, WK, WV, W_ln, B_ln, W_pz, None, H, D)
    _replay_equals_eager(lambda: tops.attn_pair_bias.forward(X, Z, pre, scale=1.0, W_proj_g=Wg, B_proj_g=None,
                                                             W_proj_o=Wo, B_proj_o=None, mask=km))


def test_triangle_attention_graph_replay(device):
    N, C, H, D = 136, 128, 4, 32
    X = rnd(N, N, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=1)
    WQ, WK, WV, Wg, Wo = (rnd(C, C, dtype=torch.bfloat16, device=device, sd=C**-0.5, seed=s) for s in range(3, 8))
    W_ln = 1.0 + rnd(C, dtype=torch.bfloat16, device=device, sd=0.1, seed=9)
    B_ln = rnd(C, dtype=torch.bfloat16, device=device, sd=0.1, seed=10)
    W_pz = rnd(C, H, dtype=torch.bfloat16, device=device, sd=C**-0.5, seed=11)
    mask = torch.rand(N, N, device=device, generator=torch.Generator(device=device).manual_seed(12)) < 0.9
    mask[5] = False  # one pair row with every key masked: the dead-row kernel writes it
    pre = tops.triangle_attn.precompute(W_ln, B_ln, WQ, WK, WV, W_pz, None, H, D)
    _replay_equals_eager(lambda: tops.triangle_attn.forward(X, pre, mask=mask, scale=D**-0.5, W_proj_g=Wg,
                                                            B_proj_g=None, W_proj_o=Wo, B_proj_o=None))
