"""Autograd operators of backend="b200" over the sm_100a C ABI.

``trop_route_hidden_b200`` mirrors ``trop_route_hidden_tilelang``
(backends/tilelang_route.py:680-727) and ``pairwise_b200`` mirrors ``pairwise_tilelang``
(backends/pairwise_tilelang.py:537-549): same positional arguments, same outputs
(``hidden, winner, margins`` / ``out, indices, margins``), route outputs marked
non-differentiable, gradients only for the float inputs. Every kernel runs on
``torch.cuda.current_stream()``; buffers come from PyTorch's caching allocator and are
handed to the kernels as raw pointers. There is no CPU path: CPU tensors raise.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import Tensor

from . import _native as nat
from . import distributed as _dist
from . import trace

__all__ = [
    "packed_route_index_dtype",
    "pairwise_anchor_index",
    "pairwise_b200",
    "trop_route_hidden_b200",
]


def packed_route_index_dtype(cells: int) -> torch.dtype:
    """Route-index packing of the reference (layers/routing.py:18-23)."""
    if cells <= 256:
        return torch.uint8
    if cells <= 32767:
        return torch.int16
    return torch.int64


def _launch(name: str, fn: Any, *args: Any) -> None:
    tr = trace.current()
    if tr is None:
        nat.check(fn(*args), name)
        return
    rec = tr.begin(name)
    status = fn(*args)
    tr.end(rec)
    nat.check(status, name)


def _require_cuda(t: Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"backend='b200' requires CUDA tensors ({what} is on {t.device}); there is no CPU fallback")


def _require_f32(t: Tensor, what: str) -> None:
    if t.dtype != torch.float32:
        raise TypeError(f"backend='b200' computes in float32; {what} has dtype {t.dtype}")


def _check_target(target: str) -> None:
    """The ``target`` keyword of the reference's TileLang wrappers (tilelang_route.py:688,
    pairwise_tilelang.py:545): a compile target. The b200 kernels are prebuilt for sm_100a,
    so any CUDA target selects them and anything else is refused."""
    if not isinstance(target, str) or not target.split()[0:1] == ["cuda"]:
        raise ValueError(f"backend='b200' runs prebuilt sm_100a kernels; target must be a CUDA target, got {target!r}")


# ---------------------------------------------------------------------------
# PairwiseLinear
# ---------------------------------------------------------------------------


def pairwise_anchor_index(anchors: Tensor, in_features: int) -> tuple[Tensor, Tensor]:
    """Inverse anchor map (feature -> anchor entries) used by the STE backward."""
    _require_cuda(anchors, "anchors")
    tables, comparisons, _ = anchors.shape
    lib = nat.load()
    anchors_c = anchors.to(dtype=torch.int64).contiguous()
    start = torch.empty(in_features + 1, device=anchors.device, dtype=torch.int32)
    entries = torch.empty(tables * comparisons * 2, device=anchors.device, dtype=torch.int32)
    with torch.cuda.device(anchors.device):
        _launch(
            "pairwise_anchor_index",
            lib.tropnn_b200_pairwise_anchor_index,
            anchors_c.data_ptr(),
            tables,
            comparisons,
            in_features,
            start.data_ptr(),
            entries.data_ptr(),
            nat.stream_handle(anchors.device),
        )
    return start, entries


def lut_grad_direct(tables: int, comparisons: int, out_features: int) -> bool:
    """Whether the LUT gradient takes the one-kernel path (tropnn_b200_pairwise_lut_grad:
    shared-memory sort + register gather per table and 64-column block) rather than the
    bucket_sort + segment_rowsum pair: up to 256 buckets, and up to 1024 columns, since every
    64-column block sorts its table's rows again (config 2: 28.7 us against 49 us; config 5's
    4096 columns: 36 ms against 16 ms)."""
    return tables >= 1 and 1 <= comparisons <= 8 and out_features <= 1024


class _PairwiseB200Function(torch.autograd.Function):
    @staticmethod
    def forward(  # type: ignore[override]
        ctx: Any,
        latent: Tensor,
        thresholds: Tensor,
        lut: Tensor,
        anchors: Tensor,
        anchor_start: Tensor,
        anchor_entries: Tensor,
        use_min_margin_ste: bool,
        surrogate: int,
        output_scale: float,
        ste: bool,
    ) -> tuple[Tensor, Tensor, Tensor]:
        batch, steps, in_features = latent.shape
        tables, comparisons, _ = anchors.shape
        out_features = lut.shape[2]
        items = batch * steps
        dev = latent.device
        latent_flat = latent.reshape(items, in_features).contiguous()
        thr = thresholds.contiguous()
        lut_c = lut.contiguous()
        out = torch.empty((items, out_features), device=dev, dtype=torch.float32)
        indices = torch.empty((items, tables), device=dev, dtype=torch.int64)
        margins = torch.empty((items, tables, comparisons), device=dev, dtype=torch.float32)
        lib = nat.load()
        _launch(
            "pairwise_forward",
            lib.tropnn_b200_pairwise_forward,
            latent_flat.data_ptr(),
            items,
            in_features,
            anchors.data_ptr(),
            thr.data_ptr(),
            nat.float_code(thr.dtype),
            tables,
            comparisons,
            lut_c.data_ptr(),
            nat.float_code(lut_c.dtype),
            out_features,
            float(output_scale),
            out.data_ptr(),
            indices.data_ptr(),
            margins.data_ptr(),
            nat.stream_handle(dev),
        )
        ctx.save_for_backward(indices, margins, anchors, lut_c, anchor_start, anchor_entries)
        ctx.shape = (batch, steps, in_features, tables, comparisons, out_features)
        ctx.use_min = bool(use_min_margin_ste)
        ctx.surrogate = int(surrogate)
        ctx.output_scale = float(output_scale)
        ctx.ste = bool(ste)
        ctx.thr_dtype = thr.dtype
        idx_out = indices.view(batch, steps, tables)
        margins_out = margins.view(batch, steps, tables, comparisons)
        ctx.mark_non_differentiable(idx_out, margins_out)
        return out.view(batch, steps, out_features), idx_out, margins_out

    @staticmethod
    def backward(ctx: Any, grad_out: Tensor, grad_idx: Tensor | None, grad_margins: Tensor | None) -> tuple[Any, ...]:
        del grad_idx, grad_margins
        indices, margins, anchors, lut, anchor_start, anchor_entries = ctx.saved_tensors
        batch, steps, in_features, tables, comparisons, out_features = ctx.shape
        items = batch * steps
        dev = grad_out.device
        g = grad_out.reshape(items, out_features).to(torch.float32).contiguous()
        stream = nat.stream_handle(dev)
        lib = nat.load()
        buckets = 1 << comparisons

        grad_lut = None
        lut_peer = _dist.fused_lut_peer() if ctx.needs_input_grad[2] else None
        if lut_peer is not None and lut_grad_direct(tables, comparisons, out_features):
            need = lut_peer.lut_capacity(tables, comparisons, out_features)
            if need < 0 or need > lut_peer.capacity or tables * ((out_features + 63) // 64) > 512:
                lut_peer = None
        else:
            lut_peer = None
        if lut_peer is not None:
            # The LUT gradient and its data-parallel average in one kernel.
            grad_lut = torch.empty_like(lut)
            buffers, world, rank, capacity = lut_peer.raw()
            _launch(
                "pairwise_lut_grad",
                lib.tropnn_b200_pairwise_lut_grad_allreduce,
                g.data_ptr(),
                items,
                out_features,
                indices.data_ptr(),
                tables,
                comparisons,
                ctx.output_scale,
                grad_lut.data_ptr(),
                nat.float_code(grad_lut.dtype),
                buffers,
                world,
                rank,
                capacity,
                1,
                stream,
            )
            _dist.mark_reduced(grad_lut)
        elif ctx.needs_input_grad[2] and lut_grad_direct(tables, comparisons, out_features):
            grad_lut = torch.empty_like(lut)
            _launch(
                "pairwise_lut_grad",
                lib.tropnn_b200_pairwise_lut_grad,
                g.data_ptr(),
                items,
                out_features,
                indices.data_ptr(),
                tables,
                comparisons,
                ctx.output_scale,
                grad_lut.data_ptr(),
                nat.float_code(grad_lut.dtype),
                stream,
            )
        elif ctx.needs_input_grad[2]:
            perm = torch.empty((tables, items), device=dev, dtype=torch.int32)
            seg = torch.empty((tables, buckets + 1), device=dev, dtype=torch.int32)
            _launch(
                "bucket_sort",
                lib.tropnn_b200_bucket_sort,
                indices.data_ptr(),
                nat.I64,
                items,
                tables,
                tables,
                buckets,
                perm.data_ptr(),
                seg.data_ptr(),
                stream,
            )
            grad_lut = torch.empty_like(lut)
            if lut.dtype in (torch.float16, torch.bfloat16) and out_features % 8 == 0 and g.data_ptr() % 16 == 0:
                # Half-precision LUT: the bucket sums gather g rounded to the LUT dtype (after a
                # power-of-two scale fitted to g's maximum, undone in the sums' epilogue), half
                # the bytes of every gathered row; the sums are rounded to that dtype anyway.
                pdt = nat.float_code(lut.dtype)
                gmax = torch.zeros(1, device=dev, dtype=torch.int32)
                _launch("absmax", lib.tropnn_b200_absmax_f32, g.data_ptr(), g.numel(), gmax.data_ptr(), stream)
                g_half = torch.empty((items, 2 * out_features), device=dev, dtype=lut.dtype)
                _launch("split_half", lib.tropnn_b200_split_half, g.data_ptr(), items, out_features, pdt,
                        gmax.data_ptr(), g_half.data_ptr(), stream)
                _launch(
                    "pairwise_lut_grad", lib.tropnn_b200_segment_rowsum_half, g_half.data_ptr(), pdt, items,
                    out_features, 2 * out_features, tables, buckets, perm.data_ptr(), seg.data_ptr(),
                    ctx.output_scale, gmax.data_ptr(), grad_lut.data_ptr(), nat.float_code(grad_lut.dtype), stream,
                )
            else:
                _launch(
                    "pairwise_lut_grad",
                    lib.tropnn_b200_segment_rowsum,
                    g.data_ptr(),
                    items,
                    out_features,
                    out_features,
                    tables,
                    buckets,
                    perm.data_ptr(),
                    seg.data_ptr(),
                    None,
                    ctx.output_scale,
                    None,
                    None,
                    None,
                    0.0,
                    1.0,
                    grad_lut.data_ptr(),
                    nat.float_code(grad_lut.dtype),
                    None,
                    stream,
                )
        # Under distributed.overlapped_gradient_sync the LUT gradient's all-reduce runs on a
        # side stream while the straight-through kernels below execute.
        pending = (
            _dist.begin_gradient_reduce(grad_lut)
            if grad_lut is not None and lut_peer is None
            else None
        )

        grad_latent = grad_thr = None
        want_latent = ctx.needs_input_grad[0]
        want_thr = ctx.needs_input_grad[1]
        if ctx.ste and (want_latent or want_thr):
            gx = torch.empty((items, in_features), device=dev, dtype=torch.float32)
            gu = torch.empty((items, tables) if ctx.use_min else (items, tables, comparisons), device=dev, dtype=torch.float32)
            rstar = torch.empty((items, tables), device=dev, dtype=torch.uint8)
            _launch(
                "pairwise_ste_backward",
                lib.tropnn_b200_pairwise_ste_backward,
                g.data_ptr(),
                items,
                out_features,
                ctx.output_scale,
                indices.data_ptr(),
                margins.data_ptr(),
                anchors.data_ptr(),
                tables,
                comparisons,
                in_features,
                lut.data_ptr(),
                nat.float_code(lut.dtype),
                int(ctx.use_min),
                ctx.surrogate,
                anchor_start.data_ptr(),
                anchor_entries.data_ptr(),
                gx.data_ptr(),
                gu.data_ptr(),
                rstar.data_ptr(),
                stream,
            )
            if want_thr:
                grad_thr = torch.empty((tables, comparisons), device=dev, dtype=ctx.thr_dtype)
                ws_bytes = lib.tropnn_b200_pairwise_threshold_grad_workspace_size(items, tables, comparisons)
                ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
                _launch(
                    "pairwise_threshold_grad",
                    lib.tropnn_b200_pairwise_threshold_grad,
                    gu.data_ptr(),
                    rstar.data_ptr(),
                    items,
                    tables,
                    comparisons,
                    int(ctx.use_min),
                    grad_thr.data_ptr(),
                    nat.float_code(ctx.thr_dtype),
                    ws.data_ptr(),
                    ws_bytes,
                    stream,
                )
            if want_latent:
                grad_latent = gx.view(batch, steps, in_features)
        _dist.end_gradient_reduce(pending, dev)
        if grad_thr is not None:
            _dist.reduce_gradient_now(grad_thr)
        return grad_latent, grad_thr, grad_lut, None, None, None, None, None, None, None


def _check_pairwise_args(latent: Tensor, anchors: Tensor, thresholds: Tensor, lut: Tensor) -> None:
    for name, t in (("latent", latent), ("anchors", anchors), ("thresholds", thresholds), ("lut", lut)):
        _require_cuda(t, name)
        if t.device != latent.device:
            raise ValueError(f"{name} is on {t.device} but latent is on {latent.device}")
    if latent.ndim != 3:
        raise ValueError(f"latent must have shape [batch, steps, in_features], got {tuple(latent.shape)}")
    _require_f32(latent, "latent")
    if anchors.ndim != 3 or anchors.shape[2] != 2:
        raise ValueError(f"anchors must have shape [tables, comparisons, 2], got {tuple(anchors.shape)}")
    if anchors.dtype != torch.int64:
        raise TypeError(f"anchors must be int64, got {anchors.dtype}")
    tables, comparisons, _ = anchors.shape
    if thresholds.shape != (tables, comparisons):
        raise ValueError(f"thresholds must have shape {(tables, comparisons)}, got {tuple(thresholds.shape)}")
    if lut.ndim != 3 or lut.shape[0] != tables or lut.shape[1] != (1 << comparisons):
        raise ValueError(f"lut must have shape [tables, 2**comparisons, out_features], got {tuple(lut.shape)}")
    nat.float_code(thresholds.dtype)
    nat.float_code(lut.dtype)


def pairwise_b200(
    latent: Tensor,
    anchors: Tensor,
    thresholds: Tensor,
    lut: Tensor,
    *,
    use_min_margin_ste: bool,
    surrogate: str = "fast_sigmoid_odd",
    target: str = "cuda",
    output_scale: float = 1.0,
    ste: bool = True,
    anchor_index: tuple[Tensor, Tensor] | None = None,
) -> tuple[Tensor, Tensor, Tensor]:
    """PairwiseLinear route + LUT sum with the STE backward, on sm_100a.

    Returns ``(out [B,S,out] f32, indices [B,S,T] int64, margins [B,S,T,C] f32)`` like
    ``pairwise_tilelang``. ``target`` is the TileLang compile target of the reference's
    signature: only CUDA targets are accepted (the kernels are prebuilt for sm_100a).
    ``output_scale`` is folded into the kernels (the ``output * output_scale`` of
    layers/base.py:76-77); ``ste=False`` drops the straight-through terms so
    ``latent``/``thresholds`` get no gradient, which is what the torch path does outside
    training (layers/pairwise.py:245).
    """
    _check_target(target)
    if surrogate not in nat.SURROGATES:
        raise ValueError(f"Pairwise b200 backend does not support surrogate={surrogate!r}")
    _check_pairwise_args(latent, anchors, thresholds, lut)
    anchors = anchors.contiguous()
    if anchor_index is None:
        anchor_index = pairwise_anchor_index(anchors, latent.shape[-1])
    start, entries = anchor_index
    with torch.cuda.device(latent.device):
        return _PairwiseB200Function.apply(
            latent,
            thresholds,
            lut,
            anchors,
            start,
            entries,
            bool(use_min_margin_ste),
            nat.SURROGATES[surrogate],
            float(output_scale),
            bool(ste),
        )


# ---------------------------------------------------------------------------
# TropLinear
# ---------------------------------------------------------------------------


def _onehot_hidden_eligible(items: int, code_dim: int, heads: int, cells: int, dtype: torch.dtype, idx: torch.dtype) -> bool:
    """Shapes the tensor-core code sum takes (tropnn_b200_trop_hidden with code_t)."""
    return (
        dtype in (torch.float16, torch.bfloat16)
        and idx == torch.uint8
        and cells in (2, 4, 8, 16, 32)
        and code_dim % 64 == 0
        and 64 <= code_dim <= 256
        and (heads * cells) % 8 == 0
        and items >= 128
    )


def _tc_backward_eligible(items: int, code_dim: int, heads: int, cells: int, dtype: torch.dtype, idx: torch.dtype) -> bool:
    """Shapes the tensor-core min-face backward takes (trop_gm / trop_router_term / trop_param_grad)."""
    return (
        dtype in (torch.float16, torch.bfloat16)
        and idx == torch.uint8
        and cells in (2, 4, 8, 16, 32)
        and code_dim % 64 == 0
        and 64 <= code_dim <= 256
        and (heads * cells) % 8 == 0
        and items >= 128
        and items % 8 == 0
    )


def _hidden_workspace(lib: Any, items: int, code_dim: int, heads: int, cells: int, dev: torch.device) -> Tensor | None:
    """Room for the slice partials of the tensor-core code sum / router term when a batch has
    too few 128-row blocks for the SMs (tropnn_b200_trop_hidden_workspace_size; None when it
    runs unsplit)."""
    nbytes = int(lib.tropnn_b200_trop_hidden_workspace_size(items, code_dim, heads, cells))
    return torch.empty(nbytes, device=dev, dtype=torch.uint8) if nbytes else None


def _param_grad_rows_eligible(param_dtype: torch.dtype, index_dtype: torch.dtype, cells: int) -> bool:
    """Layers whose code / router gradients tropnn_b200_trop_param_grad_rows sums directly."""
    return param_dtype == torch.float32 and index_dtype == torch.uint8 and 2 <= cells <= 32


def _trop_backward_tensor_cores(ctx, g, z, weight, code, winner, runner, margins, lib, stream):
    """Min-face backward as four tcgen05 GEMMs (layers/tropical_exact.py:204-237):
    gm from <g, c_r - c_w> (split-f32 g against the code table, route-picking epilogue),
    grad_latent's router term as a one-hot GEMM with +-gm weights against router_weight^T,
    and the code / router gradients as P^T X with X = g^T or z^T (one tile of 128 cells per
    CTA, the weighted one-hot P^T assembled in TMEM). grad_hidden and gm are scaled by a power
    of two fitted to grad_hidden's maximum (tropnn_b200_absmax_f32) before their rounding to the
    parameter dtype, and the results are scaled back: with f16 parameters, gradients below f16's
    range keep the precision the reference's f32 products give them."""
    batch, steps, code_dim, heads, cells = ctx.shape
    items = batch * steps
    dev = g.device
    training = ctx.training
    pdt = nat.float_code(weight.dtype)
    hk = heads * cells
    if g.data_ptr() % 16:
        g = g.clone()
    gmax = torch.zeros(1, device=dev, dtype=torch.int32)
    _launch("absmax", lib.tropnn_b200_absmax_f32, g.data_ptr(), g.numel(), gmax.data_ptr(), stream)
    gm = None
    g_t = None  # grad_hidden^T in the parameter dtype, the code gradient's operand
    if training:
        g_split = torch.empty((items, 2 * code_dim), device=dev, dtype=weight.dtype)
        if ctx.needs_input_grad[3] and items % 2 == 0:
            # The [hi | lo] split and the code gradient's transposed operand in one pass over g.
            g_t = torch.empty((code_dim, items), device=dev, dtype=weight.dtype)
            _launch("split_transpose_half", lib.tropnn_b200_split_transpose_half, g.data_ptr(), items, code_dim, pdt,
                    gmax.data_ptr(), g_split.data_ptr(), g_t.data_ptr(), stream)
        else:
            _launch("split_half", lib.tropnn_b200_split_half, g.data_ptr(), items, code_dim, pdt, gmax.data_ptr(),
                    g_split.data_ptr(), stream)
        gm = torch.empty((items, heads), device=dev, dtype=torch.float32)
        _launch(
            "trop_gm", lib.tropnn_b200_trop_gm, g_split.data_ptr(), items, code_dim, code.data_ptr(), pdt, heads, cells,
            winner.data_ptr(), runner.data_ptr(), margins.data_ptr(), ctx.code_scale, gm.data_ptr(), gmax.data_ptr(),
            stream,
        )
        w_t = torch.empty((code_dim, hk), device=dev, dtype=weight.dtype)
        _launch("trop_code_transpose", lib.tropnn_b200_trop_code_transpose, weight.data_ptr(), pdt, heads, cells, code_dim,
                w_t.data_ptr(), stream)
        grad_z = torch.empty((items, code_dim), device=dev, dtype=torch.float32)
        ws = _hidden_workspace(lib, items, code_dim, heads, cells, dev)
        _launch(
            "trop_router_term", lib.tropnn_b200_trop_router_term, g.data_ptr(), items, code_dim, w_t.data_ptr(), pdt, heads,
            cells, winner.data_ptr(), runner.data_ptr(), gm.data_ptr(), gmax.data_ptr(), grad_z.data_ptr(),
            nat.ptr(ws), 0 if ws is None else ws.numel(), stream,
        )
    else:
        grad_z = g
    grad_w = grad_b = grad_c = None
    if ctx.needs_input_grad[3]:
        if g_t is None:
            g_t = torch.empty((code_dim, items), device=dev, dtype=weight.dtype)
            _launch("transpose_to_half", lib.tropnn_b200_transpose_to_half, g.data_ptr(), nat.F32, items, code_dim,
                    pdt, gmax.data_ptr(), g_t.data_ptr(), stream)
        grad_c = torch.empty_like(code)
        _launch(
            "trop_code_grad", lib.tropnn_b200_trop_param_grad, 1 if training else 0, g_t.data_ptr(), items, code_dim, pdt,
            heads, cells, winner.data_ptr(), nat.ptr(runner), margins.data_ptr() if training else None, ctx.code_scale,
            grad_c.data_ptr(), None, gmax.data_ptr(), stream,
        )
    if training and (ctx.needs_input_grad[1] or ctx.needs_input_grad[2]):
        z_t = torch.empty((code_dim, items), device=dev, dtype=weight.dtype)
        _launch("transpose_to_half", lib.tropnn_b200_transpose_to_half, z.data_ptr(), nat.float_code(z.dtype), items,
                code_dim, pdt, None, z_t.data_ptr(), stream)
        grad_w = torch.empty_like(weight)
        grad_b = torch.empty((heads, cells), device=dev, dtype=weight.dtype)
        _launch(
            "trop_router_grad", lib.tropnn_b200_trop_param_grad, 2, z_t.data_ptr(), items, code_dim, pdt, heads, cells,
            winner.data_ptr(), runner.data_ptr(), gm.data_ptr(), 1.0, grad_w.data_ptr(), grad_b.data_ptr(),
            gmax.data_ptr(), stream,
        )
    if not ctx.needs_input_grad[1]:
        grad_w = None
    if not ctx.needs_input_grad[2]:
        grad_b = None
    return grad_z.view(batch, steps, code_dim).to(z.dtype), grad_w, grad_b, grad_c, None, None, None, None


class _TropRouteB200Function(torch.autograd.Function):
    @staticmethod
    def forward(  # type: ignore[override]
        ctx: Any,
        latent: Tensor,
        router_weight: Tensor,
        router_bias: Tensor,
        code: Tensor,
        code_scale: float,
        training: bool,
        keep_margins: bool,
        split_dtype: torch.dtype | None,
    ) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        batch, steps, code_dim = latent.shape
        heads, cells, _ = router_weight.shape
        items = batch * steps
        dev = latent.device
        z = latent.reshape(items, code_dim).contiguous()
        weight = router_weight.contiguous()
        bias = router_bias.contiguous()
        code_c = code.contiguous()
        pdt = nat.float_code(weight.dtype)
        if bias.dtype != weight.dtype or code_c.dtype != weight.dtype:
            raise TypeError("router_weight, router_bias and code must share one dtype on backend='b200'")
        idx_dtype = packed_route_index_dtype(cells)
        # Packed routes only; the runner-up and the margins exist only when the min-face
        # mix (training) or the caller (debug cache) needs them.
        winner = torch.empty((items, heads), device=dev, dtype=idx_dtype)
        runner = torch.empty((items, heads), device=dev, dtype=idx_dtype) if training else None
        margins = torch.empty((items, heads) if (training or keep_margins) else (0,), device=dev, dtype=torch.float32)
        hidden = torch.empty((items, code_dim), device=dev, dtype=torch.float32)
        # The output map's [hi | lo] operand, written by the code sum's epilogue (no separate
        # split pass over hidden).
        split = torch.empty((items, 2 * code_dim) if split_dtype is not None else (0,), device=dev,
                            dtype=split_dtype if split_dtype is not None else code_c.dtype)
        stream = nat.stream_handle(dev)
        lib = nat.load()
        icode = nat.index_code(idx_dtype)
        zcode = nat.float_code(z.dtype)
        # The tensor-core route reads the bias in f32 (exact upcast of the parameter).
        bias_in = bias if bias.dtype == torch.float32 else bias.float()
        # f32 latent and parameters: room for the split operands of the 3xTF32 tensor-core route.
        route_ws_bytes = int(lib.tropnn_b200_trop_route_workspace_size(items, code_dim, heads, cells, zcode, pdt))
        route_ws = torch.empty(route_ws_bytes, device=dev, dtype=torch.uint8) if route_ws_bytes else None
        _launch(
            "trop_route",
            lib.tropnn_b200_trop_route,
            z.data_ptr(),
            zcode,
            items,
            code_dim,
            weight.data_ptr(),
            bias_in.data_ptr(),
            nat.F32,
            pdt,
            heads,
            cells,
            None,
            winner.data_ptr(),
            nat.ptr(runner),
            icode,
            margins.data_ptr() if margins.numel() else None,
            nat.ptr(route_ws),
            route_ws_bytes,
            stream,
        )
        # Half-precision codes: the selected-code sum runs as a one-hot tensor-core GEMM
        # over code^T (rebuilt every call: code may have changed in place, and the
        # transpose is one pass over the table).
        code_t = None
        if _onehot_hidden_eligible(items, code_dim, heads, cells, code_c.dtype, idx_dtype):
            code_t = torch.empty((code_dim, heads * cells), device=dev, dtype=code_c.dtype)
            _launch(
                "trop_code_transpose",
                lib.tropnn_b200_trop_code_transpose,
                code_c.data_ptr(),
                pdt,
                heads,
                cells,
                code_dim,
                code_t.data_ptr(),
                stream,
            )
        hidden_ws = _hidden_workspace(lib, items, code_dim, heads, cells, dev) if code_t is not None else None
        _launch(
            "trop_hidden",
            lib.tropnn_b200_trop_hidden,
            z.data_ptr(),
            zcode,
            items,
            code_dim,
            code_c.data_ptr(),
            nat.ptr(code_t),
            pdt,
            heads,
            cells,
            winner.data_ptr(),
            nat.ptr(runner),
            icode,
            margins.data_ptr() if margins.numel() else None,
            float(code_scale),
            int(bool(training)),
            hidden.data_ptr(),
            split.data_ptr() if split.numel() else None,
            nat.ptr(hidden_ws),
            0 if hidden_ws is None else hidden_ws.numel(),
            stream,
        )
        ctx.save_for_backward(z, weight, code_c, winner, runner, margins)
        ctx.code_scale = float(code_scale)
        ctx.training = bool(training)
        ctx.shape = (batch, steps, code_dim, heads, cells)
        winner_out = winner.view(batch, steps, heads)
        margins_out = margins.view(batch, steps, heads) if margins.dim() == 2 else margins
        ctx.mark_non_differentiable(winner_out, margins_out, split)
        return hidden.view(batch, steps, code_dim), winner_out, margins_out, split

    @staticmethod
    def backward(
        ctx: Any, grad_hidden: Tensor, grad_winner: Tensor | None, grad_margins: Tensor | None, grad_split: Tensor | None
    ) -> tuple[Any, ...]:
        del grad_winner, grad_margins, grad_split
        z, weight, code, winner, runner, margins = ctx.saved_tensors
        batch, steps, code_dim, heads, cells = ctx.shape
        items = batch * steps
        dev = grad_hidden.device
        training = ctx.training
        g = grad_hidden.reshape(items, code_dim).to(torch.float32).contiguous()
        stream = nat.stream_handle(dev)
        lib = nat.load()
        pdt = nat.float_code(weight.dtype)
        icode = nat.index_code(winner.dtype)

        if _tc_backward_eligible(items, code_dim, heads, cells, weight.dtype, winner.dtype):
            return _trop_backward_tensor_cores(ctx, g, z, weight, code, winner, runner, margins, lib, stream)

        coef_w = coef_r = gm = None
        if training and items > 0:
            grad_z = torch.empty((items, code_dim), device=dev, dtype=torch.float32)
            coef_w = torch.empty((items, heads), device=dev, dtype=torch.float32)
            coef_r = torch.empty((items, heads), device=dev, dtype=torch.float32)
            gm = torch.empty((items, heads), device=dev, dtype=torch.float32)
            _launch(
                "trop_backward_rows",
                lib.tropnn_b200_trop_backward_rows,
                g.data_ptr(),
                items,
                code_dim,
                weight.data_ptr(),
                code.data_ptr(),
                pdt,
                heads,
                cells,
                winner.data_ptr(),
                runner.data_ptr(),
                icode,
                margins.data_ptr(),
                ctx.code_scale,
                1,
                grad_z.data_ptr(),
                coef_w.data_ptr(),
                coef_r.data_ptr(),
                gm.data_ptr(),
                stream,
            )
        else:
            # Eval: the output does not depend on the routes' margins, so grad_latent is the
            # incoming gradient and every winner code gets code_scale * g (coefficient constant).
            grad_z = g
        want_code = ctx.needs_input_grad[3]
        want_router = training and (ctx.needs_input_grad[1] or ctx.needs_input_grad[2])
        grad_w = grad_b = grad_c = None
        if (want_code or want_router) and items > 0 and _param_grad_rows_eligible(weight.dtype, winner.dtype, cells):
            # f32 parameters, u8 routes, up to 32 cells: the batch sums straight from the rows.
            grad_c = torch.empty_like(code) if want_code else None
            if want_router:
                grad_w = torch.empty_like(weight)
                grad_b = torch.empty((heads, cells), device=dev, dtype=weight.dtype)
            z32 = z if z.dtype == torch.float32 else z.float()
            _launch(
                "trop_param_grad_rows", lib.tropnn_b200_trop_param_grad_rows, g.data_ptr(), z32.data_ptr(), items,
                code_dim, pdt, heads, cells, winner.data_ptr(), nat.ptr(runner) if training else None, icode,
                nat.ptr(coef_w), nat.ptr(coef_r) if training else None, ctx.code_scale, nat.ptr(gm),
                nat.ptr(grad_c), nat.ptr(grad_w), nat.ptr(grad_b), stream,
            )
        elif (want_code or want_router) and items > 0:
            perm_w = torch.empty((heads, items), device=dev, dtype=torch.int32)
            seg_w = torch.empty((heads, cells + 1), device=dev, dtype=torch.int32)
            _launch(
                "bucket_sort",
                lib.tropnn_b200_bucket_sort,
                winner.data_ptr(),
                icode,
                items,
                heads,
                heads,
                cells,
                perm_w.data_ptr(),
                seg_w.data_ptr(),
                stream,
            )
            perm_r = seg_r = None
            if training:
                perm_r = torch.empty((heads, items), device=dev, dtype=torch.int32)
                seg_r = torch.empty((heads, cells + 1), device=dev, dtype=torch.int32)
                _launch(
                    "bucket_sort",
                    lib.tropnn_b200_bucket_sort,
                    runner.data_ptr(),
                    icode,
                    items,
                    heads,
                    heads,
                    cells,
                    perm_r.data_ptr(),
                    seg_r.data_ptr(),
                    stream,
                )
            if want_code:
                grad_c = torch.empty_like(code)
                _launch(
                    "trop_code_grad",
                    lib.tropnn_b200_segment_rowsum,
                    g.data_ptr(),
                    items,
                    code_dim,
                    code_dim,
                    heads,
                    cells,
                    perm_w.data_ptr(),
                    seg_w.data_ptr(),
                    nat.ptr(coef_w),
                    1.0 if training else ctx.code_scale,
                    nat.ptr(perm_r),
                    nat.ptr(seg_r),
                    nat.ptr(coef_r),
                    1.0,
                    1.0,
                    grad_c.data_ptr(),
                    pdt,
                    None,
                    stream,
                )
            if want_router:
                grad_w = torch.empty_like(weight)
                grad_b = torch.empty((heads, cells), device=dev, dtype=weight.dtype)
                z32 = z if z.dtype == torch.float32 else z.float()
                _launch(
                    "trop_router_grad",
                    lib.tropnn_b200_segment_rowsum,
                    z32.data_ptr(),
                    items,
                    code_dim,
                    code_dim,
                    heads,
                    cells,
                    perm_w.data_ptr(),
                    seg_w.data_ptr(),
                    gm.data_ptr(),
                    1.0,
                    perm_r.data_ptr(),
                    seg_r.data_ptr(),
                    gm.data_ptr(),
                    -1.0,
                    1.0,
                    grad_w.data_ptr(),
                    pdt,
                    grad_b.data_ptr(),
                    stream,
                )
        elif want_code:
            grad_c = torch.zeros_like(code)
        if want_router and grad_w is None:
            grad_w = torch.zeros_like(weight)
            grad_b = torch.zeros((heads, cells), device=dev, dtype=weight.dtype)
        if not ctx.needs_input_grad[1]:
            grad_w = None
        if not ctx.needs_input_grad[2]:
            grad_b = None
        # A half-precision latent gets its gradient rounded once to its dtype, as the
        # reference's `.to(compute_dtype)` backward does.
        return grad_z.view(batch, steps, code_dim).to(z.dtype), grad_w, grad_b, grad_c, None, None, None, None


def trop_route_hidden_b200(
    latent: Tensor,
    router_weight: Tensor,
    router_bias: Tensor,
    code: Tensor,
    *,
    code_scale: float,
    training: bool = False,
    target: str = "cuda",
    score_route_max_bytes: int | None = None,
) -> tuple[Tensor, Tensor, Tensor]:
    """TropLinear route + selected-code sum with the min-face backward, on sm_100a.

    ``router_weight``/``code`` ``[H, K, D]`` and ``router_bias`` ``[H, K]`` share one float
    dtype (f32/f16/bf16, upcast in-kernel). ``latent`` ``[B, S, D]`` is f32, or the
    parameters' half dtype: then the route scores run on the tensor cores (tcgen05) when
    the shape allows, with exact products of the half-precision operands and f32
    accumulation. Returns ``(hidden [B,S,D] f32, winner [B,S,H] int64, margins [B,S,H]
    f32)`` like ``trop_route_hidden_tilelang``. In eval mode (``training=False``) the output
    does not depend on the margins, so router gradients are ``None`` as in the torch path.
    ``target`` (a CUDA compile target) and ``score_route_max_bytes`` (the reference's cap on
    materialised score chunks, tilelang_route.py:689) are accepted for signature parity; the
    fused kernels materialise no scores, so the cap only has to be valid.
    """
    _check_target(target)
    if score_route_max_bytes is not None and score_route_max_bytes < 0:
        raise ValueError(f"score_route_max_bytes must be >= 0 when set, got {score_route_max_bytes}")
    hidden, winner, margins = trop_route_hidden_packed(
        latent, router_weight, router_bias, code, code_scale=code_scale, training=training, keep_margins=True
    )
    return hidden, winner.to(torch.int64), margins


def trop_route_hidden_packed(
    latent: Tensor,
    router_weight: Tensor,
    router_bias: Tensor,
    code: Tensor,
    *,
    code_scale: float,
    training: bool = False,
    keep_margins: bool = True,
) -> tuple[Tensor, Tensor, Tensor]:
    """``trop_route_hidden_b200`` with the winners in the packed route dtype (uint8 for
    cells <= 256, layers/routing.py:18-23) instead of int64, and the margins computed in
    eval only when ``keep_margins`` (otherwise an empty tensor). The layers use it so the
    int64 debug-cache copy of the routes is made only when someone reads it."""
    hidden, winner, margins, _ = trop_route_hidden_split(
        latent, router_weight, router_bias, code, code_scale=code_scale, training=training, keep_margins=keep_margins
    )
    return hidden, winner, margins


def trop_route_hidden_split(
    latent: Tensor,
    router_weight: Tensor,
    router_bias: Tensor,
    code: Tensor,
    *,
    code_scale: float,
    training: bool = False,
    keep_margins: bool = True,
    split_dtype: torch.dtype | None = None,
) -> tuple[Tensor, Tensor, Tensor, Tensor | None]:
    """``trop_route_hidden_packed`` that also returns hidden's [hi | lo] split in
    ``split_dtype`` ([items, 2 * code_dim], hi = half(hidden), lo = half(hidden - hi)): the left
    operand of the output map's f32-input product (``linear_f32out_b200(..., hidden_split=)``),
    formed by the code sum's epilogue. ``split_dtype`` must be the code dtype (f16/bf16); None
    returns no split."""
    for name, t in (("latent", latent), ("router_weight", router_weight), ("router_bias", router_bias), ("code", code)):
        _require_cuda(t, name)
        if t.device != latent.device:
            raise ValueError(f"{name} is on {t.device} but latent is on {latent.device}")
    if latent.ndim != 3:
        raise ValueError(f"latent must have shape [batch, steps, code_dim], got {tuple(latent.shape)}")
    if router_weight.ndim != 3:
        raise ValueError(f"router_weight must have shape [heads, cells, code_dim], got {tuple(router_weight.shape)}")
    if router_bias.shape != router_weight.shape[:2]:
        raise ValueError(f"router_bias must have shape [heads, cells], got {tuple(router_bias.shape)}")
    if code.shape != router_weight.shape:
        raise ValueError(f"code must match router_weight shape, got {tuple(code.shape)} and {tuple(router_weight.shape)}")
    if latent.shape[-1] != router_weight.shape[-1]:
        raise ValueError(f"latent code_dim {latent.shape[-1]} does not match router_weight code_dim {router_weight.shape[-1]}")
    if latent.dtype not in (torch.float32, router_weight.dtype):
        raise TypeError(
            f"backend='b200' latent must be float32 or the parameter dtype {router_weight.dtype}, got {latent.dtype}"
        )
    if not math.isfinite(float(code_scale)):
        raise ValueError(f"code_scale must be finite, got {code_scale}")
    if split_dtype is not None and (split_dtype != code.dtype or split_dtype not in (torch.float16, torch.bfloat16)
                                    or latent.shape[-1] % 4 != 0):
        raise ValueError(f"split_dtype {split_dtype} needs f16/bf16 codes of that dtype and code_dim % 4 == 0")
    with torch.cuda.device(latent.device):
        hidden, winner, margins, split = _TropRouteB200Function.apply(
            latent, router_weight, router_bias, code, float(code_scale), bool(training), bool(keep_margins), split_dtype
        )
    return hidden, winner, margins, (split if split_dtype is not None else None)


# in_features the exact eval path routes on: the fp32 route kernel stages a row of x per lane in
# shared memory (32 rows x (in + 4) floats within 200 KiB).
EXACT_EVAL_MAX_IN = 1536


def trop_exact_eval_b200(
    x: Tensor,
    router_eff: Tensor,
    router_bias: Tensor,
    value_eff: Tensor,
    base_out: Tensor,
    *,
    code_scale: float,
    keep_margins: bool = True,
) -> tuple[Tensor, Tensor, Tensor]:
    """TropLinear's ``exact_fused="eval"`` forward (layers/tropical_exact.py:297-358) on sm_100a,
    given its effective weights: the route kernel scores x [N, in] against router_eff
    [H, K, in] (+ router_bias, fp32 FMA) and keeps the top-2; the code-sum kernel adds
    code_scale * sum_h value_eff[h, winner] [H, K, out] onto base_out = x base^T + b [N, out].
    Returns (y [N, out] f32, winner [N, H] in the packed route dtype, margins [N, H] f32, or
    empty without ``keep_margins``). Inference only: no autograd."""
    for name, t in (("x", x), ("router_eff", router_eff), ("router_bias", router_bias), ("value_eff", value_eff),
                    ("base_out", base_out)):
        _require_cuda(t, name)
        _require_f32(t, name)
        if t.device != x.device:
            raise ValueError(f"{name} is on {t.device} but x is on {x.device}")
    items, in_features = x.shape
    heads, cells, _ = router_eff.shape
    out_features = value_eff.shape[2]
    if router_eff.shape[2] != in_features or router_bias.shape != (heads, cells) or value_eff.shape[:2] != (heads, cells):
        raise ValueError("trop_exact_eval_b200: effective weight shapes do not match")
    if base_out.shape != (items, out_features):
        raise ValueError(f"base_out must have shape {(items, out_features)}, got {tuple(base_out.shape)}")
    if in_features > EXACT_EVAL_MAX_IN:
        raise ValueError(f"trop_exact_eval_b200 routes on at most {EXACT_EVAL_MAX_IN} input features, got {in_features}")
    dev = x.device
    idx_dtype = packed_route_index_dtype(cells)
    winner = torch.empty((items, heads), device=dev, dtype=idx_dtype)
    margins = torch.empty((items, heads) if keep_margins else (0,), device=dev, dtype=torch.float32)
    y = torch.empty((items, out_features), device=dev, dtype=torch.float32)
    xs, w, b, v, base = (t.contiguous() for t in (x, router_eff, router_bias, value_eff, base_out))
    lib = nat.load()
    icode = nat.index_code(idx_dtype)
    with torch.cuda.device(dev):
        stream = nat.stream_handle(dev)
        _launch("trop_route", lib.tropnn_b200_trop_route, xs.data_ptr(), nat.F32, items, in_features, w.data_ptr(),
                b.data_ptr(), nat.F32, nat.F32, heads, cells, None, winner.data_ptr(), None, icode,
                margins.data_ptr() if margins.numel() else None, None, 0, stream)
        _launch("trop_hidden", lib.tropnn_b200_trop_hidden, base.data_ptr(), nat.F32, items, out_features, v.data_ptr(),
                None, nat.F32, heads, cells, winner.data_ptr(), None, icode, None, float(code_scale), 0, y.data_ptr(),
                None, None, 0, stream)
    return y, winner, margins


def linear_f32out_shape_ok(out_features: int, in_features: int) -> bool:
    """Weight shapes [out, in] the tensor-core f32-input linear map tiles."""
    return in_features % 64 == 0 and 64 <= in_features <= 256 and out_features % 4 == 0


def linear_f32out_eligible(hidden: Tensor, weight: Tensor) -> bool:
    """Shapes the tensor-core f32-input linear map takes (tropnn_b200_linear_f32out)."""
    out_features, in_features = weight.shape
    return (
        hidden.is_cuda
        and hidden.dtype == torch.float32
        and weight.dtype in (torch.float16, torch.bfloat16)
        and linear_f32out_shape_ok(out_features, in_features)
        and hidden.shape[-1] == in_features
    )


def linear_grad_eligible(rows: int, out_features: int, in_features: int) -> bool:
    """Shapes the tensor-core output-map gradients take (tropnn_b200_linear_dgrad / _wgrad)."""
    return rows >= 1 and out_features % 32 == 0 and in_features % 32 == 0 and 32 <= in_features <= 256


class _LinearF32OutFunction(torch.autograd.Function):
    """F.linear(hidden, weight.float(), bias.float()) for f32 ``hidden`` and half-precision
    parameters (layers/tropical.py:140-146). Forward: hidden split into [hi | lo] halves and
    one tcgen05 GEMM (two k slices against the same weight tile, bias in the epilogue).
    Backward: the reference's f32 products (grad_hidden = g W, grad_W = g^T hidden, grad_b
    = sum g) as tcgen05 tf32 GEMMs with split operands (f32 accuracy and range), grad_W and
    grad_b cast back to the parameter dtypes like the reference's ``.to`` upcast."""

    @staticmethod
    def forward(ctx: Any, hidden: Tensor, weight: Tensor, bias: Tensor | None, hidden_split: Tensor | None) -> Tensor:
        rows, in_features = hidden.shape
        out_features = weight.shape[0]
        dev = hidden.device
        h = hidden.contiguous()
        w = weight.contiguous()
        dcode = nat.float_code(w.dtype)
        stream = nat.stream_handle(dev)
        lib = nat.load()
        if hidden_split is not None:
            split = hidden_split  # formed by the producer of hidden (the code sum's epilogue)
        else:
            split = torch.empty((rows, 2 * in_features), device=dev, dtype=w.dtype)
            _launch("split_half", lib.tropnn_b200_split_half, h.data_ptr(), rows, in_features, dcode, None,
                    split.data_ptr(), stream)
        b32 = None if bias is None else bias.to(torch.float32).contiguous()
        out = torch.empty((rows, out_features), device=dev, dtype=torch.float32)
        _launch(
            "linear_f32out",
            lib.tropnn_b200_linear_f32out,
            split.data_ptr(),
            rows,
            2,
            w.data_ptr(),
            out_features,
            in_features,
            dcode,
            nat.ptr(b32),
            out.data_ptr(),
            stream,
        )
        ctx.save_for_backward(h, w)
        ctx.bias_dtype = None if bias is None else bias.dtype
        return out

    @staticmethod
    def backward(ctx: Any, grad_out: Tensor) -> tuple[Tensor | None, Tensor | None, Tensor | None, None]:
        h, w = ctx.saved_tensors
        rows, in_features = h.shape
        out_features = w.shape[0]
        dev = h.device
        g = grad_out.to(torch.float32).contiguous()
        need_b = ctx.bias_dtype is not None and ctx.needs_input_grad[2]
        if not linear_grad_eligible(rows, out_features, in_features):
            # Widths the tf32 gradient kernels do not tile: the reference's f32 products.
            return (
                g @ w.to(torch.float32) if ctx.needs_input_grad[0] else None,
                (g.t() @ h).to(w.dtype) if ctx.needs_input_grad[1] else None,
                g.sum(0).to(ctx.bias_dtype) if need_b else None,
                None,
            )
        stream = nat.stream_handle(dev)
        lib = nat.load()
        grad_h = grad_w = grad_b = None
        if ctx.needs_input_grad[0]:
            w32 = w.to(torch.float32).contiguous()
            grad_h = torch.empty((rows, in_features), device=dev, dtype=torch.float32)
            ws_bytes = int(lib.tropnn_b200_linear_dgrad_workspace_size(rows, out_features, in_features))
            ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
            _launch(
                "linear_dgrad", lib.tropnn_b200_linear_dgrad, g.data_ptr(), rows, out_features, w32.data_ptr(),
                in_features, grad_h.data_ptr(), nat.ptr(ws), ws_bytes, stream,
            )
        if ctx.needs_input_grad[1] or need_b:
            h_big = torch.empty_like(h)
            h_small = torch.empty_like(h)
            _launch("tf32_split", lib.tropnn_b200_tf32_split, h.data_ptr(), h.numel(), h_big.data_ptr(),
                    h_small.data_ptr(), stream)
            gw = torch.empty_like(w)
            gb = torch.empty((out_features,), device=dev, dtype=torch.float32) if need_b else None
            _launch(
                "linear_wgrad", lib.tropnn_b200_linear_wgrad, g.data_ptr(), rows, out_features, h_big.data_ptr(),
                h_small.data_ptr(), in_features, nat.float_code(w.dtype), gw.data_ptr(), nat.ptr(gb), stream,
            )
            grad_w = gw if ctx.needs_input_grad[1] else None
            grad_b = gb.to(ctx.bias_dtype) if need_b else None
        return grad_h, grad_w, grad_b, None


def linear_f32out_b200(
    hidden: Tensor, weight: Tensor, bias: Tensor | None, hidden_split: Tensor | None = None
) -> Tensor:
    """f32 ``hidden`` [..., in] times the half-precision ``weight`` [out, in] (+ bias) in f32.
    ``hidden_split`` (optional): hidden's [hi | lo] split [rows, 2 * in] in the weight dtype,
    as ``trop_route_hidden_split`` returns it; without it the split is formed here."""
    if not linear_f32out_eligible(hidden, weight):
        raise ValueError(
            f"linear_f32out_b200: unsupported hidden {tuple(hidden.shape)} {hidden.dtype} / weight "
            f"{tuple(weight.shape)} {weight.dtype}"
        )
    rows = hidden.numel() // max(hidden.shape[-1], 1)
    if hidden_split is not None and (
        hidden_split.dtype != weight.dtype
        or tuple(hidden_split.shape) != (rows, 2 * hidden.shape[-1])
        or not hidden_split.is_contiguous()
        or hidden_split.device != hidden.device
    ):
        raise ValueError(
            f"linear_f32out_b200: hidden_split {tuple(hidden_split.shape)} {hidden_split.dtype} does not match "
            f"hidden {tuple(hidden.shape)} and weight {weight.dtype}"
        )
    lead = hidden.shape[:-1]
    with torch.cuda.device(hidden.device):
        out = _LinearF32OutFunction.apply(hidden.reshape(-1, hidden.shape[-1]), weight, bias, hidden_split)
    return out.reshape(*lead, weight.shape[0])


# ---------------------------------------------------------------------------
# TropLinear input projection
# ---------------------------------------------------------------------------


def proj_eligible(x: Tensor, weight: Tensor) -> bool:
    """Shapes the tensor-core projection takes (tropnn_b200_trop_proj): f32 input, f16/bf16
    weight [code_dim, in] with code_dim in {64, 128, 192, 256} and in a multiple of 8."""
    code_dim, in_features = weight.shape
    return (
        x.is_cuda
        and x.dtype == torch.float32
        and weight.dtype in (torch.float16, torch.bfloat16)
        and code_dim in (64, 128, 192, 256)
        and in_features % 8 == 0
        and x.shape[-1] == in_features
    )


def _launch_proj(x: Tensor, weight: Tensor) -> Tensor:
    rows, in_features = x.shape
    code_dim = weight.shape[0]
    dev = x.device
    lib = nat.load()
    z = torch.empty((rows, code_dim), device=dev, dtype=weight.dtype)
    ws_bytes = int(lib.tropnn_b200_trop_proj_workspace_size(rows, in_features, code_dim))
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
    _launch(
        "trop_proj", lib.tropnn_b200_trop_proj, x.data_ptr(), rows, in_features, weight.data_ptr(),
        nat.float_code(weight.dtype), code_dim, z.data_ptr(), nat.ptr(ws), ws_bytes, nat.stream_handle(dev),
    )
    return z


class _TropProjFunction(torch.autograd.Function):
    """z = proj(x.to(P.dtype)) (layers/tropical.py:96-99) for a half-precision P: forward on
    the tcgen05 projection kernel (x rounded on chip, f32 accumulation, z rounded to P's dtype).
    Backward of the reference's half-precision F.linear: grad_x = grad_z P on the tcgen05
    linear map (f32 result; the reference rounds it to P's dtype and back, a difference below
    that dtype's rounding), grad_P = grad_z^T half(x) on the tcgen05 weight-gradient kernel
    (x rounded on chip; cuBLAS only for batches that are not a multiple of 8 rows)."""

    @staticmethod
    def forward(ctx: Any, x: Tensor, weight: Tensor) -> Tensor:
        xc = x.contiguous()
        w = weight.contiguous()
        z = _launch_proj(xc, w)
        ctx.save_for_backward(xc, w)
        return z

    @staticmethod
    def backward(ctx: Any, grad_z: Tensor) -> tuple[Tensor | None, Tensor | None]:
        x, w = ctx.saved_tensors
        rows, in_features = x.shape
        code_dim = w.shape[0]
        dev = x.device
        g = grad_z.to(w.dtype).contiguous()
        lib = nat.load()
        stream = nat.stream_handle(dev)
        grad_x = grad_w = None
        if ctx.needs_input_grad[0]:
            pdt = nat.float_code(w.dtype)
            w_t = torch.empty((in_features, code_dim), device=dev, dtype=w.dtype)
            _launch("trop_code_transpose", lib.tropnn_b200_trop_code_transpose, w.data_ptr(), pdt, code_dim, 1,
                    in_features, w_t.data_ptr(), stream)
            grad_x = torch.empty((rows, in_features), device=dev, dtype=torch.float32)
            _launch("linear_f32out", lib.tropnn_b200_linear_f32out, g.data_ptr(), rows, 1, w_t.data_ptr(),
                    in_features, code_dim, pdt, None, grad_x.data_ptr(), stream)
        if ctx.needs_input_grad[1]:
            if rows % 8 == 0:
                # grad_P = g^T half(x) on the tensor cores, x rounded on chip (no cast pass).
                pdt = nat.float_code(w.dtype)
                g_t = torch.empty((code_dim, rows), device=dev, dtype=w.dtype)
                _launch("transpose_to_half", lib.tropnn_b200_transpose_to_half, g.data_ptr(), pdt, rows, code_dim, pdt,
                        None, g_t.data_ptr(), stream)
                grad_w = torch.empty_like(w)
                ws_bytes = int(lib.tropnn_b200_trop_proj_wgrad_workspace_size(rows, in_features, code_dim))
                ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
                _launch("trop_proj_wgrad", lib.tropnn_b200_trop_proj_wgrad, x.data_ptr(), rows, in_features,
                        g_t.data_ptr(), pdt, code_dim, grad_w.data_ptr(), nat.ptr(ws), ws_bytes, stream)
            else:
                # Batches whose transposed gradient rows are not 16-byte multiples: the library GEMM.
                grad_w = g.t().matmul(x.to(w.dtype))
        return grad_x, grad_w


def trop_project_b200(x: Tensor, weight: Tensor) -> Tensor:
    """``proj(x.to(weight.dtype))`` for f32 ``x`` [..., in] and a half-precision ``weight``
    [code_dim, in], on the tensor-core projection kernel; returns z [..., code_dim] in the
    weight's dtype."""
    if not proj_eligible(x, weight):
        raise ValueError(
            f"trop_project_b200: unsupported x {tuple(x.shape)} {x.dtype} / weight {tuple(weight.shape)} {weight.dtype}"
        )
    lead = x.shape[:-1]
    with torch.cuda.device(x.device):
        z = _TropProjFunction.apply(x.reshape(-1, x.shape[-1]), weight)
    return z.reshape(*lead, weight.shape[0])


# ---------------------------------------------------------------------------
# f32 linear maps on the tensor cores (3xTF32)
# ---------------------------------------------------------------------------


def _ceil4(n: int) -> int:
    return (n + 3) // 4 * 4


def gemm_f32_eligible(*mats: Tensor) -> bool:
    """f32 CUDA matrices whose rows the tensor-core f32 product can read with TMA: contiguous,
    16-byte aligned, a row length that is a multiple of 4 floats."""
    return all(
        t.is_cuda and t.dtype == torch.float32 and t.dim() == 2 and t.is_contiguous() and t.shape[1] % 4 == 0
        and t.data_ptr() % 16 == 0
        for t in mats
    )


def gemm_f32(a: Tensor, b: Tensor, bias: Tensor | None = None, *, k: int | None = None, n: int | None = None) -> Tensor:
    """C = A B^T (+ bias) for f32 A [m, >=k] and B [>=n, >=k] (row strides = their widths),
    on the 3xTF32 tensor-core kernel (tropnn_b200_gemm_tf32x3); returns C [m, n] f32."""
    m = a.shape[0]
    k = a.shape[1] if k is None else k
    n = b.shape[0] if n is None else n
    dev = a.device
    c = torch.empty((m, n), device=dev, dtype=torch.float32)
    bias_c = None if bias is None else bias.to(torch.float32).contiguous()
    lib = nat.load()
    ws_bytes = int(lib.tropnn_b200_gemm_tf32x3_workspace_size(m, n, k))
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
    _launch("gemm_tf32x3", lib.tropnn_b200_gemm_tf32x3, a.data_ptr(), a.shape[1], b.data_ptr(), b.shape[1], m,
            n, k, nat.ptr(bias_c), c.data_ptr(), n, nat.ptr(ws), ws_bytes, nat.stream_handle(dev))
    return c


def transpose_f32(x: Tensor, pad_to: int = 4) -> Tensor:
    """x^T for an f32 [rows, cols] matrix, as [cols, ldo] with ldo = rows rounded up to
    ``pad_to`` and the padding columns zero (tropnn_b200_transpose_f32)."""
    rows, cols = x.shape
    ldo = (rows + pad_to - 1) // pad_to * pad_to
    out = torch.empty((cols, ldo), device=x.device, dtype=torch.float32)
    _launch("transpose_f32", nat.load().tropnn_b200_transpose_f32, x.data_ptr(), rows, cols, x.shape[1],
            out.data_ptr(), ldo, nat.stream_handle(x.device))
    return out


def _padded_cols(x: Tensor) -> Tensor:
    """x [rows, n] with its rows padded with zeros to a multiple of 4 floats (TMA row stride)."""
    n = x.shape[1]
    if n % 4 == 0:
        return x.contiguous()
    return torch.nn.functional.pad(x, (0, _ceil4(n) - n)).contiguous()


class _LinearF32Function(torch.autograd.Function):
    """F.linear(x, weight, bias) in f32 (the reference's f32 projection and output map,
    layers/tropical.py:96-99, :140-146) on the 3xTF32 tensor-core product, forward and
    backward: y = x W^T + b, grad_x = g W, grad_W = g^T x, grad_b = sum_n g."""

    @staticmethod
    def forward(ctx: Any, x: Tensor, weight: Tensor, bias: Tensor | None) -> Tensor:
        xc = x.contiguous()
        w = weight.contiguous()
        y = gemm_f32(xc, w, bias)
        ctx.save_for_backward(xc, w)
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx: Any, grad_y: Tensor) -> tuple[Tensor | None, Tensor | None, Tensor | None]:
        x, w = ctx.saved_tensors
        rows, in_features = x.shape
        out_features = w.shape[0]
        g = grad_y.to(torch.float32).contiguous()
        grad_x = grad_w = grad_b = None
        if ctx.needs_input_grad[0]:
            # grad_x = g W: B = W^T [in, out] (row stride padded to 4 floats).
            grad_x = gemm_f32(_padded_cols(g), transpose_f32(w), k=out_features, n=in_features)
        if ctx.needs_input_grad[1]:
            # grad_W = g^T x: A = g^T [out, rows], B = x^T [in, rows].
            grad_w = gemm_f32(transpose_f32(g), transpose_f32(x), k=rows, n=in_features)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            grad_b = torch.empty(out_features, device=g.device, dtype=torch.float32)
            _launch("colsum_f32", nat.load().tropnn_b200_colsum_f32, g.data_ptr(), rows, out_features, out_features,
                    grad_b.data_ptr(), nat.stream_handle(g.device))
        return grad_x, grad_w, grad_b


def linear_f32_eligible(x: Tensor, weight: Tensor) -> bool:
    """Shapes the f32 tensor-core linear map takes: f32 CUDA input and weight with an input
    width that is a multiple of 4."""
    return (
        x.is_cuda
        and x.dtype == torch.float32
        and weight.dtype == torch.float32
        and weight.dim() == 2
        and x.shape[-1] == weight.shape[1]
        and weight.shape[1] % 4 == 0
    )


def linear_f32_b200(x: Tensor, weight: Tensor, bias: Tensor | None) -> Tensor:
    """``F.linear(x, weight, bias)`` in f32 on the tensor cores (3xTF32), with its backward."""
    if not linear_f32_eligible(x, weight):
        raise ValueError(f"linear_f32_b200: unsupported x {tuple(x.shape)} {x.dtype} / weight {tuple(weight.shape)}")
    lead = x.shape[:-1]
    with torch.cuda.device(x.device):
        y = _LinearF32Function.apply(x.reshape(-1, x.shape[-1]), weight, bias)
    return y.reshape(*lead, weight.shape[0])
