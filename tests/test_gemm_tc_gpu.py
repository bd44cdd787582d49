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


@pytest.mark.parametrize("m,n,k,bias,gelu,residual,masked", [
    (1, 256, 256, False, False, False, False), (1000, 768, 256, False, False, False, False),
    (1000, 1024, 256, True, True, False, False), (1000, 256, 1024, True, False, True, True),
    (4100, 128, 256, True, False, False, False), (777, 512, 768, True, True, False, False),
    (30001, 256, 256, False, False, True, True),
    # K = 256 with many row blocks and no residual or GELU: the weight-
    # stationary kernel (N = 256, 512, 768; ragged last row block)
    (80001, 256, 256, True, False, False, True), (80000, 512, 256, True, False, False, False),
    (150017, 768, 256, False, False, False, True)])
def test_gemm_general_epilogue_matches_torch(m, n, k, bias, gelu, residual, masked):
    """kernels.gemm at the model's projection shapes: bias, GELU, residual add
    and dead-row zeroing, N = 128 (tile width 128) and multiples of 256."""
    from graph_rewrite_system_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    b = torch.randn(n, device=DEV, generator=g) if bias else None
    r = torch.randn(m, n, device=DEV, generator=g).to(torch.bfloat16) if residual else None
    live = (torch.rand(m, device=DEV, generator=g) > 0.3) if masked else None
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    out = K.gemm(x, w, b, gelu=gelu, residual=r, zero_row=live, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = x.float() @ w.float().T
    if b is not None:
        ref = ref + b
    if r is not None:
        ref = ref + r.float()
    if gelu:
        ref = torch.nn.functional.gelu(ref)
    if live is not None:
        ref = ref * live.unsqueeze(1)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("m,rows_per_beam", [(1000, 10), (20000, 250)])
def test_gemm_layernorm_masks_match_torch(m, rows_per_beam):
    """gemm_layernorm with the live-node update's masks: affinity row scale,
    rows of dead slots or inactive beams keep their input, rows of beams with
    no history keep it too, dead rows zeroed."""
    from graph_rewrite_system_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(m)
    k = 512
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    b = torch.randn(256, device=DEV, generator=g)
    res = torch.randn(m, 256, device=DEV, generator=g).to(torch.bfloat16)
    gamma = torch.randn(256, device=DEV, generator=g)
    beta = torch.randn(256, device=DEV, generator=g)
    beams = m // rows_per_beam
    scale = torch.rand(m, device=DEV, generator=g)
    where_row = torch.rand(m, device=DEV, generator=g) > 0.2
    where_beam = torch.rand(beams, device=DEV, generator=g) > 0.2
    lengths = torch.randint(0, 3, (beams,), device=DEV, generator=g, dtype=torch.int32)
    zero_row = torch.rand(m, device=DEV, generator=g) > 0.1
    out = torch.full((m, 256), float("nan"), device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    K.gemm_layernorm(x, w, b, res, gamma, beta, out=out, row_scale=scale, zero_row=zero_row,
                     where_row=where_row, where_beam=where_beam, where_len=lengths,
                     rows_per_beam=rows_per_beam, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    s = res.float() + scale.unsqueeze(1) * (x.float() @ w.float().T + b)
    ref = torch.nn.functional.layer_norm(s, (256,), gamma, beta, eps=1e-5)
    beam = torch.arange(m, device=DEV) // rows_per_beam
    keep = ~(where_row & where_beam[beam] & (lengths[beam] > 0))
    ref = torch.where(keep.unsqueeze(1), res.float(), ref) * zero_row.unsqueeze(1)
    err = (out.float() - ref).abs().max().item()
    assert err <= 3e-2 * max(1.0, ref.abs().max().item()), err
    assert torch.equal(out[keep & zero_row], res[keep & zero_row])


@pytest.mark.parametrize("m,ns", [(5, 31), (37000, 31), (1000, 32), (999, 7)])
def test_match_logits_gemm_matches_torch(m, ns):
    from graph_rewrite_system_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(m + ns)
    x = torch.randn(m, 256, device=DEV, generator=g).to(torch.bfloat16)
    w = torch.zeros(32, 256, device=DEV)
    w[:ns] = torch.randn(ns, 256, device=DEV, generator=g) / 16
    w = w.to(torch.bfloat16)
    bias = torch.randn(ns, device=DEV, generator=g)
    first = torch.randint(0, 8, (ns,), device=DEV, generator=g)
    live = torch.rand(m, device=DEV, generator=g) > 0.2
    types = torch.randint(-1, 8, (m,), device=DEV, generator=g)
    logits = torch.empty(m, ns, device=DEV)
    eligible = torch.empty(m, ns, device=DEV, dtype=torch.bool)
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    K.match_logits_gemm(x, w, bias, first, live, types, 0.125, logits, eligible, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    exp_e = live.unsqueeze(1) & (types.unsqueeze(1) == first.unsqueeze(0))
    assert torch.equal(eligible, exp_e)
    ref = (x.float() @ w[:ns].float().T) * 0.125 + bias
    ref = ref.masked_fill(~exp_e, -1e4)
    assert (logits - ref).abs().max().item() <= 1e-2 * max(1.0, ref[exp_e].abs().max().item())


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


def test_graphed_token_step_rekeys_on_cache_capacity():
    """Two caches at one address with different page counts (views of one
    buffer, as a cache allocated where a freed one lived would be): the
    second must not replay the graph captured for the first, whose page-id
    bound is the smaller capacity.  Pages past the first capacity are used."""
    import bench

    search, _ = bench.build_rollout(DEV, beam_size=8, depth=4)
    model, cache = search.model, search.cache
    g = torch.Generator(device=DEV).manual_seed(5)
    W, cols, page = model.width, 4, cache.page_size
    layers, heads, hd = cache.keys.shape[0], cache.keys.shape[3], cache.keys.shape[4]
    big = 64
    kbuf = torch.randn(layers, big, page, heads, hd, device=DEV, generator=g).to(cache.keys.dtype)
    vbuf = torch.randn(layers, big, page, heads, hd, device=DEV, generator=g).to(cache.keys.dtype)
    b = 6
    ctx = torch.randn(b, 3 * W, device=DEV, generator=g).to(model.compute_dtype)
    active = torch.ones(b, device=DEV, dtype=torch.bool)
    lengths = torch.full((b,), cols * page - 3, device=DEV, dtype=torch.int32)
    for cap in (16, big):
        keys, values = kbuf[:, :cap], vbuf[:, :cap]
        assert keys.data_ptr() == kbuf.data_ptr()
        table = torch.randint(cap // 2, cap, (b, cols), device=DEV, generator=g, dtype=torch.int32)
        eager = [t.clone() for t in model._token_step_eager(ctx, active, lengths, table, keys,
                                                            values)]
        graphed = model._token_step(ctx, active, lengths, table, keys, values)
        torch.cuda.synchronize()
        for a, z in zip(eager, graphed):
            scale = max(1.0, a.float().abs().max().item())
            assert (a.float() - z.float()).abs().max().item() <= 1e-2 * scale, cap


@pytest.mark.parametrize("m,masked", [(1, False), (300, True), (4097, True), (40000, True)])
def test_graph_mlp_matches_torch(m, masked):
    """The fused graph-layer update (GELU activation kept in shared memory)
    against the torch fp32 composition of the same layer, model.py:26-53:
    LayerNorm(x + GELU([x | agg] U0^T + b0) U2^T + b2) * live."""
    from graph_rewrite_system_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(m + 3)
    a = torch.randn(m, 512, device=DEV, generator=g).to(torch.bfloat16)
    u0 = (torch.randn(512, 512, device=DEV, generator=g) / 512 ** 0.5).to(torch.bfloat16)
    u2 = (torch.randn(256, 512, device=DEV, generator=g) / 512 ** 0.5).to(torch.bfloat16)
    b0 = torch.randn(512, device=DEV, generator=g) * 0.1
    b2 = torch.randn(256, device=DEV, generator=g) * 0.1
    gamma = 1 + 0.1 * torch.randn(256, device=DEV, generator=g)
    beta = 0.1 * torch.randn(256, device=DEV, generator=g)
    live = (torch.rand(m, device=DEV, generator=g) > 0.25) if masked else None
    out_buf = torch.full((m, 512), float("nan"), device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    K.graph_mlp(a, u0, b0, u2, b2, a[:, :256], gamma, beta, zero_row=live,
                out=out_buf[:, :256], status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    x = a[:, :256].float()
    hidden = torch.nn.functional.gelu(a.float() @ u0.float().T + b0)
    s = x + hidden.to(torch.bfloat16).float() @ u2.float().T + b2
    ref = torch.nn.functional.layer_norm(s, (256,), gamma, beta, eps=1e-5)
    if live is not None:
        ref = ref * live.unsqueeze(1)
    err = (out_buf[:, :256].float() - ref).abs().max().item()
    assert err <= 3e-2 * max(1.0, ref.abs().max().item()), err
    assert torch.isnan(out_buf[:, 256:].float()).all()          # right half untouched


def test_gemm_layernorm_width_128_matches_torch():
    from graph_rewrite_system_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(128)
    m, k = 5000, 256
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(128, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    b = torch.randn(128, device=DEV, generator=g)
    res = torch.randn(m, 128, device=DEV, generator=g).to(torch.bfloat16)
    gamma = torch.randn(128, device=DEV, generator=g)
    beta = torch.randn(128, device=DEV, generator=g)
    live = torch.rand(m, device=DEV, generator=g) > 0.2
    out = torch.empty(m, 128, device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    K.gemm_layernorm(x, w, b, res, gamma, beta, out=out, zero_row=live, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    s = res.float() + x.float() @ w.float().T + b
    ref = torch.nn.functional.layer_norm(s, (128,), gamma, beta, eps=1e-5) * live.unsqueeze(1)
    err = (out.float() - ref).abs().max().item()
    assert err <= 3e-2 * max(1.0, ref.abs().max().item()), err
