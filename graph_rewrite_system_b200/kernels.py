"""Thin typed wrappers over the model kernels of libgrs_b200.so.

Each function takes torch CUDA tensors, checks the layout it needs and calls
one C-ABI entry point on the current stream.  bf16 projections run on the
library's tcgen05 GEMM (``gemm``, ``gemm_layernorm``, ``match_logits_gemm``);
``linear`` is the fp32 form used by the CPU-equivalence configuration.
"""
from __future__ import annotations

import torch

from . import _lib




def dtype_code(t: torch.Tensor) -> int:
    try:
        return _lib.DTYPE_CODES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported activation dtype {t.dtype}") from None


def stream() -> int:
    """Raw handle of the stream the wrappers launch on: the stream pinned by
    an enclosing ``pinned_stream()`` block, else torch's current stream."""
    return _lib.current_stream()


pinned_stream = _lib.pinned_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _row_stride(t: torch.Tensor) -> int:
    if t.stride(-1) != 1:
        raise ValueError("rows must be contiguous in their last dimension")
    return t.stride(-2) if t.dim() >= 2 else t.shape[-1]


def linear(x: torch.Tensor, weight_t: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """x [M, K] @ weight_t [K, N] (+ bias), fp32 (the CPU-equivalence
    configuration); bf16 activations go through ``gemm``."""
    if x.dtype != torch.float32:
        raise ValueError("bf16 projections run on the tensor-core GEMM (kernels.gemm)")
    if bias is None:
        return torch.mm(x, weight_t, out=out)
    return torch.addmm(bias, x, weight_t, out=out)


def _gemm_operands(x: torch.Tensor, weight: torch.Tensor):
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("the tensor-core GEMM takes bf16 operands")
    if x.dim() != 2 or weight.dim() != 2 or x.shape[1] != weight.shape[1]:
        raise ValueError(f"gemm shapes {tuple(x.shape)} x {tuple(weight.shape)}^T do not match")
    if x.stride(1) != 1 or weight.stride(1) != 1:
        raise ValueError("gemm operands need contiguous rows")


def gemm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
         gelu: bool = False, residual: torch.Tensor | None = None,
         zero_row: torch.Tensor | None = None, out: torch.Tensor | None = None,
         status: torch.Tensor | None = None) -> torch.Tensor:
    """out = (x @ weight.T (+ bias) (+ residual)) then GELU when `gelu`, rows
    with zero_row == 0 zeroed; one tcgen05 GEMM launch (bf16 in and out, fp32
    accumulation).  weight is a K-major [N, K] Linear weight, bias fp32 [N].
    Shapes the kernel does not take raise; there is no other path."""
    _gemm_operands(x, weight)
    m, n = x.shape[0], weight.shape[0]
    if out is None:
        out = torch.empty(m, n, device=x.device, dtype=torch.bfloat16)
    if m == 0:
        return out
    if residual is not None and (residual.shape != (m, n) or residual.dtype != torch.bfloat16):
        raise ValueError("residual must be bf16 [M, N]")
    _lib.check(_lib.lib().grs_gemm_bf16(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), m, n, x.shape[1],
        _p(bias), int(gelu), _p(residual), 0 if residual is None else _row_stride(residual),
        _p(zero_row), out.data_ptr(), _row_stride(out), _p(status), stream()), "tensor-core GEMM")
    return out


def gemm_layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                   residual: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, *,
                   out: torch.Tensor, row_scale: torch.Tensor | None = None,
                   zero_row: torch.Tensor | None = None, where_row: torch.Tensor | None = None,
                   where_beam: torch.Tensor | None = None, where_len: torch.Tensor | None = None,
                   rows_per_beam: int = 1, status: torch.Tensor | None = None,
                   eps: float = 1e-5) -> torch.Tensor:
    """out = LayerNorm(residual + row_scale * (x @ weight.T + bias)) over
    256- or 128-column rows, with the row kernels' masks: rows whose where_row /
    where_beam is 0 or whose where_len <= 0 keep `residual`, rows whose
    zero_row is 0 are zeroed.  One tcgen05 GEMM launch."""
    _gemm_operands(x, weight)
    m, n = x.shape[0], weight.shape[0]
    if n not in (128, 256) or residual.shape != (m, n) or out.shape != (m, n):
        raise ValueError("gemm_layernorm normalises [M, 256] or [M, 128] rows")
    if m == 0:
        return out
    _lib.check(_lib.lib().grs_gemm_bf16_layernorm_ex(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), m, n, x.shape[1],
        bias.data_ptr(), _p(row_scale), residual.data_ptr(), _row_stride(residual),
        gamma.data_ptr(), beta.data_ptr(), _p(zero_row), _p(where_row), _p(where_beam),
        _p(where_len), rows_per_beam, eps, out.data_ptr(), _row_stride(out), _p(status),
        stream()), "tensor-core GEMM + LayerNorm")
    return out


def graph_mlp(x: torch.Tensor, u0: torch.Tensor, b0: torch.Tensor, u2: torch.Tensor,
              b2: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
              *, out: torch.Tensor, zero_row: torch.Tensor | None = None,
              status: torch.Tensor | None = None, eps: float = 1e-5) -> torch.Tensor:
    """One InitialGraphLayer update, width 256, in one tcgen05 launch:
    out = LayerNorm(residual + GELU(x @ u0.T + b0) @ u2.T + b2), rows with
    zero_row == 0 zeroed; x = [states | aggregated messages] [M, 512]."""
    _gemm_operands(x, u0)
    m = x.shape[0]
    if (x.shape[1] != 512 or u0.shape != (512, 512) or u2.shape != (256, 512)
            or residual.shape != (m, 256) or out.shape != (m, 256)):
        raise ValueError("graph_mlp is the width-256 graph layer update")
    if m == 0:
        return out
    _lib.check(_lib.lib().grs_graph_mlp_bf16(
        x.data_ptr(), x.stride(0), u0.data_ptr(), u0.stride(0), b0.data_ptr(), u2.data_ptr(),
        u2.stride(0), b2.data_ptr(), m, residual.data_ptr(), _row_stride(residual),
        gamma.data_ptr(), beta.data_ptr(), _p(zero_row), eps, out.data_ptr(), _row_stride(out),
        _p(status), stream()), "fused graph-layer MLP")
    return out


def match_logits_gemm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                      first_types: torch.Tensor, live: torch.Tensor, types: torch.Tensor,
                      scale: float, logits: torch.Tensor, eligible: torch.Tensor,
                      status: torch.Tensor | None = None) -> None:
    """Match logits of x [M, K] against the source-vector x retrieval_node
    product weight [32, K] (rows past the source count zero) in one tcgen05
    launch: fp32 logits [M, sources] masked to -1e4 off the eligible pairs,
    eligible [M, sources]."""
    _gemm_operands(x, weight)
    m, ns = x.shape[0], first_types.numel()
    if weight.shape[0] != 32 or ns > 32:
        raise ValueError("match_logits_gemm takes at most 32 sources")
    if m == 0:
        return
    _lib.check(_lib.lib().grs_match_logits_bf16(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), m, x.shape[1], ns,
        bias.data_ptr(), first_types.data_ptr(), live.data_ptr(), types.data_ptr(), scale,
        logits.data_ptr(), eligible.data_ptr(), _p(status), stream()), "tensor-core match logits")


def add_layernorm(x, y=None, *, scale=None, gamma=None, beta=None, sum_out=None, ln_out=None,
                  zero_row=None, zero_beam=None, where_row=None, where_beam=None,
                  where_len=None, rows_per_beam=1, zero_before=False, eps=1e-5):
    rows = x.shape[0]
    width = x.shape[-1]
    _lib.check(_lib.lib().grs_add_layernorm(
        dtype_code(x), x.data_ptr(), _row_stride(x), _p(y), 0 if y is None else _row_stride(y),
        _p(scale), _p(gamma), _p(beta), _p(sum_out), 0 if sum_out is None else _row_stride(sum_out),
        _p(ln_out), 0 if ln_out is None else _row_stride(ln_out), _p(zero_row), _p(zero_beam),
        _p(where_row), _p(where_beam), _p(where_len), rows, rows_per_beam, width, eps,
        int(zero_before), stream()), "add_layernorm")


def bias_gelu(y: torch.Tensor, bias: torch.Tensor | None, gelu: bool = True) -> torch.Tensor:
    _lib.check(_lib.lib().grs_bias_gelu(dtype_code(y), y.data_ptr(), y.shape[0], y.shape[1],
                                        _row_stride(y), _p(bias), int(gelu), stream()), "bias_gelu")
    return y


def embed_initial(types, gate_emb, marker, states, live):
    rows = types.numel()
    _lib.check(_lib.lib().grs_embed_initial(dtype_code(states), types.data_ptr(), rows,
                                            states.shape[-1], gate_emb.data_ptr(), marker.data_ptr(),
                                            states.data_ptr(), _row_stride(states), live.data_ptr(),
                                            stream()), "embed_initial")


def graph_aggregate(fb, rel, ports, slots, agg):
    """ports: (in_node, in_port, out_node, out_port) int32 [B, port_slots, 4]."""
    in_node, in_port, out_node, out_port = ports
    _lib.check(_lib.lib().grs_graph_aggregate(
        dtype_code(fb), fb.data_ptr(), _row_stride(fb), rel.data_ptr(), in_node.data_ptr(),
        in_port.data_ptr(), out_node.data_ptr(), out_port.data_ptr(), fb.shape[0], slots,
        in_node.shape[1], agg.shape[-1], agg.data_ptr(), _row_stride(agg), stream()),
        "graph_aggregate")


def action_inputs(states, xfer_ids, source_ids, source_slots, xfer_emb, source_reps, bound,
                  ctx_in, source_mask, active):
    b, s, w = states.shape
    _lib.check(_lib.lib().grs_action_inputs(
        dtype_code(states), states.data_ptr(), states.stride(1), s, xfer_ids.data_ptr(),
        source_ids.data_ptr(), source_slots.data_ptr(), source_slots.shape[1], w,
        xfer_emb.data_ptr(), source_reps.data_ptr(), bound.data_ptr(), ctx_in.data_ptr(),
        source_mask.data_ptr(), active.data_ptr(), b, stream()), "action_inputs")


def position_token(raw, position, lengths, active, token):
    _lib.check(_lib.lib().grs_position_token(dtype_code(raw), raw.data_ptr(), position.data_ptr(),
                                             lengths.data_ptr(), active.data_ptr(),
                                             token.data_ptr(), raw.shape[0], raw.shape[1],
                                             stream()), "position_token")


def update_live_hidden(qxa, keys, vw, cvec, source_mask, slots, width, hidden, affinity):
    _lib.check(_lib.lib().grs_update_live_hidden(
        dtype_code(qxa), qxa.data_ptr(), _row_stride(qxa), keys.data_ptr(), vw.data_ptr(),
        cvec.data_ptr(), source_mask.data_ptr(), source_mask.shape[1], qxa.shape[0], slots, width,
        hidden.data_ptr(), _row_stride(hidden), affinity.data_ptr(), stream()), "update_live_hidden")


def destination_hidden(r, type_table, pos_table, dest_slots, dest_types, active, hidden):
    b, pattern = dest_slots.shape
    _lib.check(_lib.lib().grs_destination_hidden(
        dtype_code(r), r.data_ptr(), type_table.data_ptr(), pos_table.data_ptr(),
        dest_slots.data_ptr(), dest_types.data_ptr(), active.data_ptr(), pattern, b,
        r.shape[1], hidden.data_ptr(), stream()), "destination_hidden")


def apply_slots(states, live, types, source_slots, source_mask, dest_slots, dest_types, active,
                created):
    b, s, w = states.shape
    _lib.check(_lib.lib().grs_apply_slots(
        dtype_code(states), states.data_ptr(), states.stride(1), live.data_ptr(), types.data_ptr(),
        s, source_slots.data_ptr(), source_mask.data_ptr(), source_slots.shape[1],
        dest_slots.data_ptr(), dest_types.data_ptr(), active.data_ptr(), dest_slots.shape[1],
        created.data_ptr(), w, b, stream()), "apply_slots")


def match_logits(acc, source_bias, first_types, live, types, inv_sqrt_r, logits, eligible):
    rows = acc.shape[0]
    _lib.check(_lib.lib().grs_match_logits(
        dtype_code(acc), acc.data_ptr(), _row_stride(acc), source_bias.data_ptr(),
        first_types.data_ptr(), live.data_ptr(), types.data_ptr(), rows, first_types.numel(),
        inv_sqrt_r, logits.data_ptr(), eligible.data_ptr(), stream()), "match_logits")


def gather_beams(src: torch.Tensor, index: torch.Tensor, out: torch.Tensor, fill_byte: int = 0):
    """out[i] = src[index[i]] over the leading dim; trailing dims may differ in
    their second size (slot padding), filled with fill_byte."""
    rows = out.shape[0]
    in_bytes = src[0].numel() * src.element_size() if src.shape[0] else 0
    out_bytes = out[0].numel() * out.element_size() if rows else 0
    if not src.is_contiguous() or not out.is_contiguous():
        raise ValueError("gather_beams needs contiguous tensors")
    _lib.check(_lib.lib().grs_gather_beams(src.data_ptr(), out.data_ptr(), index.data_ptr(), rows,
                                           in_bytes, out_bytes, fill_byte, stream()),
               "gather_beams")
    return out


def edges_to_ports(edge_batch, edge_src, edge_dst, edge_relation, batch, slots, device):
    shape = (batch, slots, 4)
    ports = [torch.full(shape, -1, device=device, dtype=torch.int32) for _ in range(4)]
    out_node, out_port, in_node, in_port = ports
    e = edge_batch.numel()
    if e:
        conv = lambda t: t.to(device=device, dtype=torch.int64).contiguous()
        eb, es, ed, er = map(conv, (edge_batch, edge_src, edge_dst, edge_relation))
        _lib.check(_lib.lib().grs_edges_to_ports(eb.data_ptr(), es.data_ptr(), ed.data_ptr(),
                                                 er.data_ptr(), e, slots, out_node.data_ptr(),
                                                 out_port.data_ptr(), in_node.data_ptr(),
                                                 in_port.data_ptr(), stream()), "edges_to_ports")
    return in_node, in_port, out_node, out_port




def select_candidates(logits, eligible, distance, k, groups, out_batch, out_source, out_anchor,
                      out_prob, out_score=None):
    b, s, ns = logits.shape
    near, far = groups["near"], groups["far"]
    _lib.check(_lib.lib().grs_select_candidates(
        logits.data_ptr(), eligible.data_ptr(), distance.data_ptr(), b, s, ns, k,
        float(near["scale"]), float(near["bias"]), float(near["raw_threshold"]),
        float(far["scale"]), float(far["bias"]), float(far["raw_threshold"]),
        out_batch.data_ptr(), out_source.data_ptr(), out_anchor.data_ptr(), out_prob.data_ptr(),
        _p(out_score), stream()), "select_candidates")


def structural_decode(types, live, ports, rules, batch_ids, sources, anchors, bindings, valid,
                      clear_invalid=False):
    """rules: dict of the model's int64 rule buffers."""
    in_node, in_port, out_node, out_port = ports
    slots = types.shape[1]
    pe = rules["pattern_edges"]
    _lib.check(_lib.lib().grs_structural_decode(
        types.data_ptr(), live.data_ptr(), slots, out_node.data_ptr(), out_port.data_ptr(),
        in_node.data_ptr(), in_port.data_ptr(), rules["source_types"].data_ptr(),
        rules["source_lengths"].data_ptr(), rules["binding_child"].data_ptr(),
        rules["binding_parent"].data_ptr(), rules["binding_parent_port"].data_ptr(),
        rules["binding_child_port"].data_ptr(), rules["binding_direction"].data_ptr(),
        pe.data_ptr(), pe.shape[1], bindings.shape[1], batch_ids.data_ptr(), sources.data_ptr(),
        anchors.data_ptr(), sources.numel(), bindings.data_ptr(), valid.data_ptr(),
        int(clear_invalid), stream()), "structural_decode")


def rows_copy(segments, n_max: int, n_dev: torch.Tensor | None = None) -> None:
    """One launch of grs_rows_copy.  Each segment is (src, src_row_stride,
    src_unit_stride, src_index, dst, dst_row_stride, dst_unit_stride,
    dst_index, unit_bytes, units); src/dst are tensors (their data pointers
    are the bases), indexes int64 tensors or None, strides in bytes.  Rows:
    min(n_dev, n_max) with a device count, else n_max."""
    import numpy as np

    words = []
    for (src, sr, su, si, dst, dr, du, di, ub, units) in segments:
        if ub == 0:
            continue
        words.extend((src.data_ptr(), sr, su, 0 if si is None else si.data_ptr(),
                      dst.data_ptr(), dr, du, 0 if di is None else di.data_ptr(), ub, units))
    table = np.asarray(words, dtype=np.int64)
    _lib.check(_lib.lib().grs_rows_copy(
        len(words) // 10, table.ctypes.data if len(words) else None,
        _p(n_dev), n_max, stream()), "rows_copy")


def gemm_bias_gelu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                   gelu: bool, out: torch.Tensor, status: torch.Tensor | None = None) -> int:
    """out = (x @ weight.T (+ bias)) then GELU on the tensor cores in one
    pass (bf16; weight is a K-major [N, K] Linear weight).  Returns the
    library status: GRS_ERR_SHAPE (-4) when the shapes do not fit the kernel,
    in which case nothing was launched."""
    return _lib.lib().grs_gemm_bf16_epilogue(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), x.shape[0],
        weight.shape[0], x.shape[1], _p(bias), int(gelu), out.data_ptr(), out.stride(0),
        _p(status), stream())


def gemm_residual_layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                            residual: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                            zero_row: torch.Tensor | None, out: torch.Tensor,
                            status: torch.Tensor | None = None, eps: float = 1e-5) -> int:
    """out = LayerNorm(residual + x @ weight.T + bias) * gamma + beta (rows
    with zero_row == 0 zeroed) on the tensor cores in one pass; weight is a
    K-major [256, K] Linear weight, bf16.  Returns the library status
    (GRS_ERR_SHAPE, -4, when nothing was launched)."""
    return _lib.lib().grs_gemm_bf16_layernorm(
        x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), x.shape[0], x.shape[1],
        bias.data_ptr(), residual.data_ptr(), residual.stride(0), gamma.data_ptr(),
        beta.data_ptr(), _p(zero_row), eps, out.data_ptr(), out.stride(0), _p(status),
        stream())
