"""Decode steps replayed from CUDA graphs (MLADecodeLayer(cuda_graphs=True))
give the eager step's bits, and read their inputs live: a replay after the
inputs change in place equals an eager step on the new inputs."""
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qcau_b200 import _lib
    from qcau_b200.mla import MLAConfig, MLADecodeLayer, make_paged_cache, precompute_freqs_cis


def test_graph_replay_matches_eager():
    cfg = MLAConfig(n_heads=128)
    eager = MLADecodeLayer(cfg, "cuda")
    graphed = MLADecodeLayer(cfg, "cuda", cuda_graphs=True)
    eager.random_weights(seed=5)
    graphed.random_weights(seed=5)
    B, ctx = 16, 2048
    cache, table, seqlens = make_paged_cache(B, ctx, 64, 576, "cuda", seed=6)
    positions = seqlens.clone()
    freqs = precompute_freqs_cis(64, ctx + 1, cfg.rope_theta, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn(B, cfg.dc, device="cuda", generator=gen).to(torch.bfloat16)
    y_e = torch.empty(B, cfg.dim, device="cuda", dtype=torch.bfloat16)
    y_g = torch.empty_like(y_e)
    eager.forward(q, cache, table, seqlens, positions, freqs, ctx, y_e)
    graphed.forward(q, cache, table, seqlens, positions, freqs, ctx, y_g)  # capture
    assert len(graphed._graphs) == 1
    y_g.zero_()
    graphed.forward(q, cache, table, seqlens, positions, freqs, ctx, y_g)  # replay
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(y_e, y_g)
    # new query values and shorter sequences, in place: the replay reads them
    q.copy_(torch.randn(B, cfg.dc, device="cuda", generator=gen).to(torch.bfloat16))
    seqlens.sub_(torch.arange(B, device="cuda", dtype=seqlens.dtype) * 37)
    positions.copy_(seqlens)
    eager.forward(q, cache, table, seqlens, positions, freqs, ctx, y_e)
    graphed.forward(q, cache, table, seqlens, positions, freqs, ctx, y_g)
    torch.cuda.synchronize()
    assert len(graphed._graphs) == 1
    assert torch.equal(y_e, y_g)
    graphed.release_graphs()
    assert not graphed._graphs
