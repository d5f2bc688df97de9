"""PairwiseLinear backend="b200" on the GPU against the reference's golden vectors and the
numpy oracle (parity rule: indices bit-exact, values within 1e-5 relative in fp32 and
2e-2 relative with f16/bf16 parameters)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import tropnn_b200
from tests.golden_cases import build_layer, case_names, load_case, rel_err, state_arrays, tolerance
from tests.gpu_runner import run_b200

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-5


@pytest.mark.parametrize("name", case_names("pairwise"))
def test_pairwise_matches_reference_golden(name: str) -> None:
    arrays, meta = load_case(name)
    layer = build_layer(arrays, meta)
    got = run_b200(layer, arrays, meta)
    tol = tolerance(meta)
    assert rel_err(got["y"], arrays["y"]) <= tol
    assert np.array_equal(got["last_indices"], arrays["last_indices"])
    assert np.array_equal(got["last_margins"], arrays["last_margins"])
    if meta["train"]:
        assert rel_err(got["grad.x"], arrays["grad.x"]) <= tol
        for key in ("lut", "thresholds"):
            assert bool(got[f"has_grad.{key}"]) == bool(arrays[f"has_grad.{key}"])
            assert rel_err(got[f"grad.{key}"], arrays[f"grad.{key}"].astype(np.float32)) <= tol, key


def _oracle_case(layer: tropnn_b200.PairwiseLinear, x: np.ndarray, g: np.ndarray, *, ste: bool = True) -> dict:
    st = state_arrays(layer)
    fwd = oracle.pairwise_forward(x, st["anchors"], st["thresholds"], st["lut"], output_scale=layer.output_scale)
    bwd = oracle.pairwise_backward(
        g,
        fwd["indices"],
        fwd["margins"],
        st["anchors"],
        st["lut"],
        in_features=layer.in_features,
        output_scale=layer.output_scale,
        use_min_margin_ste=layer.use_min_margin_ste,
        surrogate=layer.surrogate,
        ste=ste,
    )
    return {**fwd, **{f"grad.{k}": v for k, v in bwd.items()}}


def _run(layer: tropnn_b200.PairwiseLinear, x: np.ndarray, g: np.ndarray, *, train: bool = True) -> dict:
    layer = layer.cuda().train(train)
    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    y = layer(xt)
    y.backward(torch.from_numpy(g).cuda().view_as(y))
    torch.cuda.synchronize()
    return {
        "out": y.detach().cpu().numpy().reshape(x.shape[0], -1),
        "indices": layer._last_indices.cpu().numpy().reshape(x.shape[0], -1),
        "margins": layer._last_margins.cpu().numpy().reshape(x.shape[0], layer.tables, layer.comparisons),
        "grad.x": None if xt.grad is None else xt.grad.cpu().numpy(),
        "grad.lut": None if layer.lut.grad is None else layer.lut.grad.float().cpu().numpy(),
        "grad.thresholds": None if layer.thresholds.grad is None else layer.thresholds.grad.float().cpu().numpy(),
    }


def _inputs(n: int, in_f: int, out_f: int, seed: int = 1) -> tuple[np.ndarray, np.ndarray]:
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(n, in_f, generator=gen).numpy(), torch.randn(n, out_f, generator=gen).numpy()


def _compare(got: dict, ref: dict, tol: float = FP32_TOL) -> None:
    assert np.array_equal(got["indices"], ref["indices"])
    assert np.array_equal(got["margins"], ref["margins"])
    assert rel_err(got["out"], ref["out"]) <= tol
    for key in ("grad.x", "grad.lut", "grad.thresholds"):
        if ref[key] is None:
            assert got[key] is None, key
        else:
            assert rel_err(got[key], ref[key]) <= tol, key


def test_config2_batch4096_matches_oracle() -> None:
    """Config 2 at its full batch: PairwiseLinear(256->512, T16, C6) fwd + min-margin STE bwd."""
    layer = tropnn_b200.PairwiseLinear(256, 512, tables=16, comparisons=6, seed=0)
    x, g = _inputs(4096, 256, 512)
    ref = _oracle_case(layer, x, g)
    _compare(_run(layer, x, g), ref)


@pytest.mark.parametrize("surrogate", ["fast_sigmoid_odd", "izhikevich"])
@pytest.mark.parametrize("use_min", [True, False])
def test_ste_modes_and_surrogates(surrogate: str, use_min: bool) -> None:
    layer = tropnn_b200.PairwiseLinear(64, 96, tables=24, comparisons=5, seed=3, surrogate=surrogate, use_min_margin_ste=use_min)
    with torch.no_grad():
        layer.thresholds.normal_(0.0, 0.3)
    x, g = _inputs(300, 64, 96, seed=4)
    _compare(_run(layer, x, g), _oracle_case(layer, x, g))


@pytest.mark.parametrize(
    ("in_f", "out_f", "tables", "comparisons", "n"),
    [
        (2, 1, 1, 1, 5),  # minimum sizes
        (784, 10, 136, 6, 512),  # config 4 layer 2: ragged width (scalar path)
        (128, 130, 7, 12, 33),  # maximum comparisons, ragged rows
        (300, 1000, 3, 2, 17),  # wide output, several column tiles
    ],
)
def test_shapes_and_edges(in_f: int, out_f: int, tables: int, comparisons: int, n: int) -> None:
    layer = tropnn_b200.PairwiseLinear(in_f, out_f, tables=tables, comparisons=comparisons, seed=5)
    x, g = _inputs(n, in_f, out_f, seed=6)
    _compare(_run(layer, x, g), _oracle_case(layer, x, g))


def test_empty_batch() -> None:
    layer = tropnn_b200.PairwiseLinear(16, 8, tables=4, comparisons=3).cuda()
    x = torch.empty(0, 16, device="cuda", requires_grad=True)
    y = layer(x)
    assert y.shape == (0, 1, 8)
    y.sum().backward()
    assert x.grad.shape == (0, 16)
    assert float(layer.lut.grad.abs().sum()) == 0.0


def test_three_d_input_and_f16_input_dtype() -> None:
    layer = tropnn_b200.PairwiseLinear(32, 24, tables=8, comparisons=4, seed=2).cuda()
    x = torch.randn(3, 5, 32, device="cuda").half()
    y = layer(x)
    assert y.shape == (3, 5, 24) and y.dtype == torch.float16
    assert layer._last_indices.shape == (3, 5, 8) and layer._last_indices.dtype == torch.int64
    assert layer._last_margins.shape == (3, 5, 8, 4)
    ref = oracle.pairwise_forward(
        x.float().reshape(15, 32).cpu().numpy(),
        *(t.detach().cpu().numpy() for t in (layer.anchors, layer.thresholds, layer.lut)),
        output_scale=layer.output_scale,
    )
    assert rel_err(y.detach().float().reshape(15, 24).cpu().numpy(), ref["out"]) <= 1e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_precision_parameters(dtype: torch.dtype) -> None:
    layer = tropnn_b200.PairwiseLinear(128, 256, tables=32, comparisons=8, seed=0).to(dtype)
    x, g = _inputs(257, 128, 256, seed=8)
    got = _run(layer, x, g)
    ref = _oracle_case(layer, x, g)
    assert np.array_equal(got["indices"], ref["indices"])
    for key in ("out", "grad.x", "grad.lut", "grad.thresholds"):
        assert rel_err(got[key], ref[key]) <= 2e-2, key
    assert layer.lut.grad.dtype == dtype and layer.thresholds.grad.dtype == dtype


def test_eval_mode_with_grad_gives_lut_grad_only() -> None:
    """The STE term is live only in training (layers/pairwise.py:245); eval backward gives LUT grads only."""
    layer = tropnn_b200.PairwiseLinear(64, 32, tables=8, comparisons=4, seed=1)
    x, g = _inputs(40, 64, 32)
    got = _run(layer, x, g, train=False)
    ref = _oracle_case(layer, x, g, ste=False)
    assert got["grad.x"] is None and got["grad.thresholds"] is None
    assert rel_err(got["grad.lut"], ref["grad.lut"]) <= FP32_TOL


def test_backward_is_deterministic() -> None:
    layer = tropnn_b200.PairwiseLinear(256, 512, tables=16, comparisons=6, seed=0)
    x, g = _inputs(4096, 256, 512)
    a = _run(layer, x, g)
    layer.zero_grad(set_to_none=True)
    b = _run(layer, x, g)
    for key in ("out", "grad.x", "grad.lut", "grad.thresholds"):
        assert np.array_equal(a[key], b[key]), key


def test_combined_c_abi_backward_matches_layer() -> None:
    """tropnn_b200_pairwise_backward (one C call, caller-provided workspace) equals the layer path."""
    from tropnn_b200 import _native as nat

    layer = tropnn_b200.PairwiseLinear(96, 80, tables=12, comparisons=5, seed=9)
    x, g = _inputs(200, 96, 80)
    ref = _run(layer, x, g)
    lib = nat.load()
    dev = torch.device("cuda")
    n, T, C, out_f = 200, 12, 5, 80
    idx = torch.from_numpy(ref["indices"]).to(dev).contiguous()
    u = torch.from_numpy(ref["margins"]).to(dev).contiguous()
    gt = torch.from_numpy(g).to(dev).contiguous()
    ws_bytes = lib.tropnn_b200_pairwise_backward_workspace_size(n, T, C, 96, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    gx = torch.empty(n, 96, device=dev)
    gthr = torch.empty(T, C, device=dev)
    glut = torch.empty_like(layer.lut)
    status = lib.tropnn_b200_pairwise_backward(
        gt.data_ptr(), n, out_f, layer.output_scale, idx.data_ptr(), u.data_ptr(), layer.anchors.data_ptr(), T, C, 96,
        layer.lut.data_ptr(), nat.F32, 1, 0, gx.data_ptr(), gthr.data_ptr(), nat.F32, glut.data_ptr(), ws.data_ptr(),
        ws_bytes, torch.cuda.current_stream().cuda_stream,
    )
    nat.check(status, "pairwise_backward")
    torch.cuda.synchronize()
    assert np.array_equal(gx.cpu().numpy(), ref["grad.x"])
    assert np.array_equal(gthr.cpu().numpy(), ref["grad.thresholds"])
    assert np.array_equal(glut.cpu().numpy(), ref["grad.lut"])
    with pytest.raises(RuntimeError, match="workspace"):
        nat.check(
            lib.tropnn_b200_pairwise_backward(
                gt.data_ptr(), n, out_f, 1.0, idx.data_ptr(), u.data_ptr(), layer.anchors.data_ptr(), T, C, 96,
                layer.lut.data_ptr(), nat.F32, 1, 0, gx.data_ptr(), gthr.data_ptr(), nat.F32, glut.data_ptr(),
                ws.data_ptr(), ws_bytes - 256, torch.cuda.current_stream().cuda_stream,
            ),
            "pairwise_backward",
        )


def test_invalid_arguments_raise_value_and_type_errors() -> None:
    layer = tropnn_b200.PairwiseLinear(16, 8, tables=4, comparisons=3).cuda()
    x = torch.randn(2, 1, 16, device="cuda")
    with pytest.raises(TypeError):
        tropnn_b200.pairwise_b200(x.double(), layer.anchors, layer.thresholds, layer.lut, use_min_margin_ste=True)
    with pytest.raises(ValueError):
        tropnn_b200.pairwise_b200(x, layer.anchors[:2], layer.thresholds, layer.lut, use_min_margin_ste=True)
    with pytest.raises(ValueError, match="surrogate"):
        tropnn_b200.pairwise_b200(x, layer.anchors, layer.thresholds, layer.lut, use_min_margin_ste=True, surrogate="x")
    with torch.no_grad():
        layer.anchors[0, 0, 0] = 99
    with pytest.raises(IndexError):
        layer(x)


@pytest.mark.parametrize(
    ("n", "out_f", "tables", "comparisons", "lut_dtype"),
    [
        (4096, 512, 16, 6, torch.float32),  # config 2: one group of 16 tables, two per warp
        (517, 130, 136, 6, torch.float32),  # 9 table groups (the last of 8), ragged columns and rows
        (300, 64, 20, 7, torch.float16),  # 128 buckets: groups of 12 tables
        (7, 40, 3, 2, torch.bfloat16),  # fewer tables than warps; fewer rows than row slices
        (0, 32, 8, 4, torch.float32),  # no rows: zeros
    ],
)
def test_lut_grad_kernel_matches_sorted_rowsum(n, out_f, tables, comparisons, lut_dtype) -> None:
    """tropnn_b200_pairwise_lut_grad (shared-memory partials, no sort) against the bucket_sort +
    segment_rowsum pair and a float64 scatter: f32 sums of the same terms in another order."""
    from tropnn_b200 import _native as nat
    from tropnn_b200.ops import lut_grad_direct

    assert lut_grad_direct(tables, comparisons, out_f)
    lib = nat.load()
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream().cuda_stream
    buckets = 1 << comparisons
    gen = torch.Generator().manual_seed(11)
    g = torch.randn(n, out_f, generator=gen).to(dev)
    idx = torch.randint(0, buckets, (n, tables), generator=gen).to(dev)
    scale = 0.37
    direct = torch.full((tables, buckets, out_f), float("nan"), device=dev, dtype=lut_dtype)
    nat.check(
        lib.tropnn_b200_pairwise_lut_grad(g.data_ptr(), n, out_f, idx.data_ptr(), tables, comparisons, scale,
                                          direct.data_ptr(), nat.float_code(lut_dtype), stream),
        "pairwise_lut_grad",
    )
    perm = torch.empty((tables, max(n, 1)), device=dev, dtype=torch.int32)
    seg = torch.empty((tables, buckets + 1), device=dev, dtype=torch.int32)
    nat.check(lib.tropnn_b200_bucket_sort(idx.data_ptr(), nat.I64, n, tables, tables, buckets, perm.data_ptr(),
                                          seg.data_ptr(), stream), "bucket_sort")
    sorted_sum = torch.empty_like(direct)
    nat.check(
        lib.tropnn_b200_segment_rowsum(g.data_ptr(), n, out_f, out_f, tables, buckets, perm.data_ptr(), seg.data_ptr(),
                                       None, scale, None, None, None, 0.0, 1.0, sorted_sum.data_ptr(),
                                       nat.float_code(lut_dtype), None, stream),
        "segment_rowsum",
    )
    torch.cuda.synchronize()
    exact = torch.zeros(tables, buckets, out_f, dtype=torch.float64)
    gd, ic = g.double().cpu() * scale, idx.cpu()
    for t in range(tables):
        exact[t].index_add_(0, ic[:, t], gd)
    tol = 1e-6 if lut_dtype == torch.float32 else (1e-3 if lut_dtype == torch.float16 else 8e-3)
    assert not torch.isnan(direct.float()).any()
    if n == 0:
        assert float(direct.float().abs().sum()) == 0.0
        return
    assert rel_err(direct.double().cpu().numpy(), exact.numpy()) <= tol
    assert rel_err(direct.double().cpu().numpy(), sorted_sum.double().cpu().numpy()) <= tol


@pytest.mark.parametrize(
    ("rows", "in_f", "out_f", "tables", "comparisons", "lut_dtype"),
    [
        (37, 64, 512, 16, 4, torch.float32),  # small LUT: the per-row-block kernel
        (258, 512, 4096, 64, 8, torch.float16),  # 128 MiB LUT: the staged gather, ragged last unit
        (70, 256, 2560, 64, 8, torch.float16),  # partial column chunk (2560 of 4096)
        (33, 256, 1536, 32, 8, torch.float32),  # f32 LUT, one partial 2048-column chunk
        (19, 128, 2048, 16, 10, torch.bfloat16),  # 1024-entry tables
        (20, 64, 8448, 8, 8, torch.float16),  # three column chunks, the last 256 columns wide
    ],
)
def test_forward_sum_is_table_ordered_f32(rows, in_f, out_f, tables, comparisons, lut_dtype) -> None:
    """y = out_scale * (((0 + L[0, i0]) + L[1, i1]) + ...) in f32, bit for bit, for the
    per-row-block kernel and for the staged gather of LUTs larger than L2; indices and margins
    against the oracle's routing."""
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(rows, in_f, generator=gen).cuda()
    anchors = torch.randint(0, in_f, (tables, comparisons, 2), generator=gen).cuda()
    thr = (torch.randn(tables, comparisons, generator=gen) * 0.1).cuda()
    lut = torch.randn(tables, 1 << comparisons, out_f, generator=gen).to(lut_dtype).cuda()
    scale = 0.37
    with torch.no_grad():
        y, idx, margins = tropnn_b200.ops.pairwise_b200(x.view(rows, 1, in_f), anchors, thr, lut, use_min_margin_ste=True,
                                                  output_scale=scale)
        idx = idx.view(rows, tables)
        acc = torch.zeros(rows, out_f, device="cuda")
        for t in range(tables):
            acc = acc + lut[t, idx[:, t]].float()
        expect = acc * scale
    torch.cuda.synchronize()
    assert torch.equal(y.view(rows, out_f), expect)
    ref_idx, ref_u = oracle.pairwise_indices(x.cpu().numpy(), anchors.cpu().numpy(), thr.cpu().numpy())
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    assert np.array_equal(margins.view(rows, tables, comparisons).cpu().numpy(), ref_u)


@pytest.mark.parametrize(
    ("in_f", "out_f", "tables", "comparisons", "n", "dtype", "surrogate", "use_min"),
    [
        (512, 2048, 32, 8, 203, torch.float32, "fast_sigmoid_odd", True),  # 64 MiB f32 LUT, ragged last unit
        (256, 4096, 40, 8, 77, torch.float16, "izhikevich", True),  # 80 MiB f16 LUT, full 8 KB rows
        (128, 3072, 48, 8, 9, torch.bfloat16, "fast_sigmoid_odd", True),  # 6 KB rows, one partial unit
        (64, 2048, 2, 12, 5, torch.float32, "fast_sigmoid_odd", True),  # 12 comparisons (4096-entry tables)
        (128, 2048, 40, 8, 37, torch.float32, "izhikevich", False),  # full STE: the per-row STE kernel
    ],
)
def test_staged_paths_match_oracle(in_f, out_f, tables, comparisons, n, dtype, surrogate, use_min) -> None:
    """LUTs larger than 32 MiB take the staged forward and the staged min-margin STE backward
    (the kernels of config 5): forward bit-exact routes and margins, output and every gradient
    against the oracle (1e-5 for f32 parameters, 2e-2 for half precision)."""
    layer = tropnn_b200.PairwiseLinear(in_f, out_f, tables=tables, comparisons=comparisons, seed=8, surrogate=surrogate,
                                       use_min_margin_ste=use_min)
    if dtype != torch.float32:
        layer = layer.to(dtype)
    with torch.no_grad():
        layer.thresholds.normal_(0.0, 0.3)
    x, g = _inputs(n, in_f, out_f, seed=9)
    _compare(_run(layer, x, g), _oracle_case(layer, x, g), tol=FP32_TOL if dtype == torch.float32 else 2e-2)


@pytest.mark.parametrize(
    ("rows", "width", "groups", "buckets", "vdtype", "gscale", "tol"),
    [
        (517, 2048, 6, 256, torch.float16, 1.0, 2e-3),
        (300, 1536, 4, 64, torch.bfloat16, 1.0, 1e-2),
        (257, 4096, 3, 256, torch.float16, 1e-7, 2e-3),  # far below f16's normal range: the scale keeps it
    ],
)
def test_segment_rowsum_half_matches_f32_sums(rows, width, groups, buckets, vdtype, gscale, tol) -> None:
    """tropnn_b200_segment_rowsum_half over g rounded by split_half (power-of-two scale from the
    gradient maximum) against tropnn_b200_segment_rowsum over the f32 g: within one rounding of
    the value dtype per summand."""
    from tropnn_b200 import _native as nat

    lib = nat.load()
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(rows)
    g = (torch.randn(rows, width, generator=gen) * gscale).to(dev)
    keys = torch.randint(0, buckets, (rows, groups), generator=gen).to(dev)
    stream = nat.stream_handle(dev)
    perm = torch.empty((groups, rows), device=dev, dtype=torch.int32)
    seg = torch.empty((groups, buckets + 1), device=dev, dtype=torch.int32)
    nat.check(lib.tropnn_b200_bucket_sort(keys.data_ptr(), nat.I64, rows, groups, groups, buckets, perm.data_ptr(),
                                          seg.data_ptr(), stream), "bucket_sort")
    ref = torch.empty((groups, buckets, width), device=dev)
    nat.check(lib.tropnn_b200_segment_rowsum(g.data_ptr(), rows, width, width, groups, buckets, perm.data_ptr(),
                                             seg.data_ptr(), None, 0.5, None, None, None, 0.0, 1.0, ref.data_ptr(),
                                             nat.F32, None, stream), "segment_rowsum")
    gmax = torch.zeros(1, device=dev, dtype=torch.int32)
    nat.check(lib.tropnn_b200_absmax_f32(g.data_ptr(), g.numel(), gmax.data_ptr(), stream), "absmax")
    split = torch.empty((rows, 2 * width), device=dev, dtype=vdtype)
    nat.check(lib.tropnn_b200_split_half(g.data_ptr(), rows, width, nat.float_code(vdtype), gmax.data_ptr(),
                                         split.data_ptr(), stream), "split_half")
    got = torch.full((groups, buckets, width), float("nan"), device=dev)
    nat.check(lib.tropnn_b200_segment_rowsum_half(split.data_ptr(), nat.float_code(vdtype), rows, width, 2 * width,
                                                  groups, buckets, perm.data_ptr(), seg.data_ptr(), 0.5,
                                                  gmax.data_ptr(), got.data_ptr(), nat.F32, stream),
              "segment_rowsum_half")
    torch.cuda.synchronize()
    assert torch.isfinite(got).all()
    assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) <= tol


def test_small_batch_kernels_are_bit_identical_to_the_per_row_kernels() -> None:
    """Up to 64 rows the forward runs a CTA per row (threads over the columns) and up to 256
    rows the min-margin STE does (tables split over its warps); both keep the per-row kernels'
    summation orders, so the first rows' output and grad_x of a 300-row batch (per-row kernels)
    and of those rows alone (row-CTA kernels) are equal bit for bit, and both match the
    oracle."""
    layer = tropnn_b200.PairwiseLinear(256, 512, tables=16, comparisons=6, seed=2)
    with torch.no_grad():
        layer.thresholds.normal_(0.0, 0.2)
    x, g = _inputs(300, 256, 512, seed=12)
    big = _run(layer, x, g)
    layer.zero_grad(set_to_none=True)
    small = _run(layer, x[:8], g[:8])
    assert np.array_equal(small["out"], big["out"][:8])
    assert np.array_equal(small["indices"], big["indices"][:8])
    assert np.array_equal(small["grad.x"], big["grad.x"][:8])
    _compare(small, _oracle_case(layer, x[:8], g[:8]))
