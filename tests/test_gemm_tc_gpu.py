"""The tcgen05 GEMM with a fused bias/GELU epilogue against a torch fp32
reference of the same op (bf16 inputs, fp32 accumulation, bf16 output;
tolerance 2e-2 relative to the output scale)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("m,n,k,bias,gelu", [(128, 256, 64, False, False), (300, 512, 512, True, True),
                                             (1000, 256, 256, True, False), (4097, 512, 512, True, True),
                                             (77, 256, 128, False, True), (20000, 512, 512, True, True)])
def test_gemm_epilogue_matches_torch(m, n, k, bias, gelu):
    from graph_rewrite_system_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    b = torch.randn(n, device=DEV, generator=g) if bias else None
    out = torch.full((m, n), float("nan"), device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    assert K.gemm_bias_gelu(x, w, b, gelu, out, status) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = x.float() @ w.float().T
    if b is not None:
        ref = ref + b
    if gelu:
        ref = torch.nn.functional.gelu(ref)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err


def test_gemm_epilogue_strided_rows_and_shape_refusal():
    from graph_rewrite_system_b200 import kernels as K

    x_buf = torch.randn(256, 1024, device=DEV).to(torch.bfloat16)
    x = x_buf[:, :512]                                   # row stride 1024
    w = (torch.randn(256, 512, device=DEV) / 512 ** 0.5).to(torch.bfloat16)
    out_buf = torch.zeros(256, 768, device=DEV, dtype=torch.bfloat16)
    out = out_buf[:, 256:512]
    assert K.gemm_bias_gelu(x, w, None, False, out) == 0
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T
    assert (out.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
    assert (out_buf[:, :256] == 0).all() and (out_buf[:, 512:] == 0).all()
    # shapes the kernel does not take are refused before anything launches
    assert K.gemm_bias_gelu(x[:, :100], w[:, :100], None, False, out) == -4


def test_readout_with_fused_update_matches_unfused():
    """The rollout model's readout (bf16, 4 readout graph layers whose u0
    projection + GELU run as one tensor-core pass) against the same readout
    with the library GEMM and the separate bias+GELU kernel, on the state of a
    short beam search: relative Frobenius error within bf16 tolerance."""
    import bench

    search, _ = bench.build_rollout(DEV, beam_size=32, depth=6)
    search.reset()
    for _ in range(3):
        assert search.step() is not None
    model = search.model
    args = (search.states, search.live, search.types)
    kw = dict(readout_key_cache=search.cache.readout_keys,
              readout_value_cache=search.cache.readout_values, block_table=search.block_table,
              lengths=search.lengths, ports=search.topo.ports())
    rows = search.states.shape[0] * search.states.shape[1]
    assert rows >= model.FUSED_MIN_ROWS
    fused, _, _ = model.readout_incremental(*args, **kw)
    model.FUSED_MIN_ROWS = 1 << 62
    try:
        plain, _, _ = model.readout_incremental(*args, **kw)
    finally:
        del model.FUSED_MIN_ROWS
    torch.cuda.synchronize()
    assert int(search.status.item()) == 0
    a, b = fused.float(), plain.float()
    rel = ((a - b).norm() / b.norm().clamp_min(1e-12)).item()
    assert rel < 1e-2, rel


@pytest.mark.parametrize("m,k,masked", [(128, 64, False), (300, 512, True), (4097, 512, True),
                                        (20000, 256, False)])
def test_gemm_layernorm_matches_torch(m, k, masked):
    """LayerNorm(residual + x W^T + b) * gamma + beta with dead rows zeroed,
    against torch fp32 on the same bf16 inputs (residual read with a row
    stride, output written into a strided view)."""
    from graph_rewrite_system_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(m + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    b = torch.randn(256, device=DEV, generator=g)
    res_buf = torch.randn(m, 512, device=DEV, generator=g).to(torch.bfloat16)
    res = res_buf[:, :256]
    gamma = torch.randn(256, device=DEV, generator=g)
    beta = torch.randn(256, device=DEV, generator=g)
    live = (torch.rand(m, device=DEV, generator=g) > 0.2) if masked else None
    out_buf = torch.full((m, 512), float("nan"), device=DEV, dtype=torch.bfloat16)
    out = out_buf[:, 256:]
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    assert K.gemm_residual_layernorm(x, w, b, res, gamma, beta, live, out, status) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    s = res.float() + x.float() @ w.float().T + b
    ref = torch.nn.functional.layer_norm(s, (256,), gamma, beta, eps=1e-5)
    if live is not None:
        ref = ref * live.unsqueeze(1)
    err = (out.float() - ref).abs().max().item()
    assert err <= 3e-2 * max(1.0, ref.abs().max().item()), err
    assert torch.isnan(out_buf[:, :256].float()).all()          # left half untouched


def test_graphed_token_step_matches_eager_with_eviction():
    """The per-beam token path replayed from captured CUDA graphs equals the
    eager path on the same inputs, while beam counts cycle through more
    shapes than the graph cache keeps (so graphs are evicted and captured
    again)."""
    import bench

    search, _ = bench.build_rollout(DEV, beam_size=8, depth=4)
    model, cache = search.model, search.cache
    model.GRAPH_CACHE_LIMIT = 2
    try:
        g = torch.Generator(device=DEV).manual_seed(11)
        W, cols = model.width, 4
        for b in (5, 9, 13, 5, 9, 13, 9):
            ctx = torch.randn(b, 3 * W, device=DEV, generator=g).to(model.compute_dtype)
            active = torch.rand(b, device=DEV, generator=g) > 0.2
            lengths = torch.randint(0, cols * cache.page_size, (b,), device=DEV, generator=g,
                                    dtype=torch.int32)
            table = torch.randint(0, cache.capacity, (b, cols), device=DEV, generator=g,
                                  dtype=torch.int32)
            eager = model._token_step_eager(ctx, active, lengths, table, cache.keys, cache.values)
            eager = [t.clone() for t in eager]
            graphed = model._token_step(ctx, active, lengths, table, cache.keys, cache.values)
            torch.cuda.synchronize()
            for a, z in zip(eager, graphed):
                scale = max(1.0, a.float().abs().max().item())
                assert (a.float() - z.float()).abs().max().item() <= 1e-2 * scale
            assert len(model._graphs[1]) <= 2
    finally:
        del model.GRAPH_CACHE_LIMIT
