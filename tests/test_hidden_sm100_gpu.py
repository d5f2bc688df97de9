"""The tensor-core (one-hot GEMM) code sum against the per-row gather kernel and the oracle.

tropnn_b200_trop_hidden with code_t runs sum_h code[h, route] as a tcgen05 GEMM whose left
operand is the one-hot route matrix; without code_t the same call gathers per row. In eval
both sum exactly the same f16/bf16 code values in f32 (order differs), so they agree to
1e-5 relative. In training the tensor-core path rounds the two mixing weights to the
parameter dtype: within 2e-3 (f16) / 1e-2 (bf16) relative, inside the 2e-2 half-precision
parity tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests.golden_cases import rel_err
from tropnn_b200 import _native as nat

pytestmark = pytest.mark.gpu

TRAIN_TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


def _routes(items: int, heads: int, cells: int, gen: torch.Generator) -> tuple[torch.Tensor, ...]:
    winner = torch.randint(0, cells, (items, heads), generator=gen)
    shift = torch.randint(1, cells, (items, heads), generator=gen)
    runner = (winner + shift) % cells  # distinct from the winner
    margins = torch.rand(items, heads, generator=gen) * 3.0
    return winner.to(torch.uint8), runner.to(torch.uint8), margins


def _hidden(latent, code, winner, runner, margins, code_scale, training, use_tc, workspace=True, split=None):
    lib = nat.load()
    items, code_dim = latent.shape
    heads, cells, _ = code.shape
    stream = torch.cuda.current_stream().cuda_stream
    code_t = None
    if use_tc:
        code_t = torch.empty((code_dim, heads * cells), device=code.device, dtype=code.dtype)
        nat.check(
            lib.tropnn_b200_trop_code_transpose(
                code.data_ptr(), nat.float_code(code.dtype), heads, cells, code_dim, code_t.data_ptr(), stream
            ),
            "trop_code_transpose",
        )
    hidden = torch.empty((items, code_dim), device=latent.device, dtype=torch.float32)
    ws_bytes = int(lib.tropnn_b200_trop_hidden_workspace_size(items, code_dim, heads, cells)) if use_tc and workspace else 0
    ws = torch.empty(ws_bytes, device=latent.device, dtype=torch.uint8) if ws_bytes else None
    nat.check(
        lib.tropnn_b200_trop_hidden(
            latent.data_ptr(), nat.float_code(latent.dtype), items, code_dim, code.data_ptr(), nat.ptr(code_t),
            nat.float_code(code.dtype), heads, cells, winner.data_ptr(), runner.data_ptr(), nat.U8,
            margins.data_ptr(), float(code_scale), int(training), hidden.data_ptr(), nat.ptr(split), nat.ptr(ws),
            ws_bytes, stream,
        ),
        "trop_hidden",
    )
    torch.cuda.synchronize()
    return hidden.cpu().numpy()


def _oracle_hidden(latent, code, winner, runner, margins, code_scale, training):
    z = latent.float().cpu().numpy()
    c = code.float().cpu().numpy()
    w = winner.long().cpu().numpy()
    r = runner.long().cpu().numpy()
    m = margins.cpu().numpy()
    heads = c.shape[0]
    head_ix = np.arange(heads)[None, :]
    values = c[head_ix, w]
    if training:
        values = oracle.minface_mix(values, c[head_ix, r], m)
    return (z + values.sum(axis=1, dtype=np.float32) * np.float32(code_scale)).astype(np.float32)


def _check(items, heads, cells, code_dim, dtype, training, latent_f32=False, seed=0):
    gen = torch.Generator().manual_seed(seed)
    latent = torch.randn(items, code_dim, generator=gen).to(torch.float32 if latent_f32 else dtype).cuda()
    code = (torch.randn(heads, cells, code_dim, generator=gen) * 0.5).to(dtype).cuda()
    winner, runner, margins = (t.cuda() for t in _routes(items, heads, cells, gen))
    scale = heads**-0.5
    tc = _hidden(latent, code, winner, runner, margins, scale, training, use_tc=True)
    simt = _hidden(latent, code, winner, runner, margins, scale, training, use_tc=False)
    ref = _oracle_hidden(latent, code, winner, runner, margins, scale, training)
    assert np.isfinite(tc).all()
    tol = TRAIN_TOL[dtype] if training else 1e-5
    assert rel_err(tc, simt) <= tol
    assert rel_err(tc, ref) <= tol
    assert rel_err(simt, ref) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("training", [False, True])
def test_config5_shape(dtype, training):
    """Config 5's code table: H1024, K16, D256 (256 k blocks per row block)."""
    _check(items=640, heads=1024, cells=16, code_dim=256, dtype=dtype, training=training)


@pytest.mark.parametrize("cells", [2, 4, 8, 16, 32])
def test_cells(cells):
    _check(items=256, heads=max(4, 512 // cells), cells=cells, code_dim=128, dtype=torch.float16, training=False)
    _check(items=256, heads=max(4, 512 // cells), cells=cells, code_dim=128, dtype=torch.float16, training=True)


@pytest.mark.parametrize(
    ("items", "heads", "cells", "code_dim"),
    [
        (300, 12, 16, 64),  # ragged rows, 3 k blocks with a partial last one
        (1000, 200, 8, 192),  # many row blocks, N=192
        (129, 20, 2, 64),  # one live row in the last block, 40 entries (one partial k block)
        (20000, 64, 16, 128),  # ~1 row block per CTA and more: the persistent loop
        (300, 1024, 16, 128),  # 3 row blocks: the contraction split into 16 slices, ragged rows
    ],
)
def test_ragged_shapes(items, heads, cells, code_dim):
    _check(items, heads, cells, code_dim, torch.float16, training=False)
    _check(items, heads, cells, code_dim, torch.bfloat16, training=True)


@pytest.mark.parametrize("training", [False, True])
def test_split_contraction_and_no_workspace(training):
    """5 row blocks of 256 k blocks: the contraction cut into slices summed in slice order by
    slice_reduce; without a workspace each row block takes one CTA over all its k blocks. Both
    agree with the gather kernel and with each other up to f32 summation order."""
    gen = torch.Generator().manual_seed(9)
    items, heads, cells, code_dim = 640, 1024, 16, 256
    latent = torch.randn(items, code_dim, generator=gen).half().cuda()
    code = (torch.randn(heads, cells, code_dim, generator=gen) * 0.5).half().cuda()
    winner, runner, margins = (t.cuda() for t in _routes(items, heads, cells, gen))
    scale = heads**-0.5
    split = _hidden(latent, code, winner, runner, margins, scale, training, use_tc=True)
    whole = _hidden(latent, code, winner, runner, margins, scale, training, use_tc=True, workspace=False)
    simt = _hidden(latent, code, winner, runner, margins, scale, training, use_tc=False)
    tol = TRAIN_TOL[torch.float16] if training else 1e-5
    assert rel_err(split, simt) <= tol and rel_err(whole, simt) <= tol
    assert rel_err(split, whole) <= 1e-5
    again = _hidden(latent, code, winner, runner, margins, scale, training, use_tc=True)
    assert np.array_equal(split, again)  # deterministic


def test_f32_latent():
    """F32 latent with half-precision codes (the reference's upcast z) takes the same path."""
    _check(items=512, heads=64, cells=16, code_dim=256, dtype=torch.float16, training=False, latent_f32=True)


def test_code_transpose():
    gen = torch.Generator().manual_seed(3)
    code = torch.randn(37, 8, 96, generator=gen).half().cuda()
    out = torch.empty(96, 37 * 8, dtype=torch.float16, device="cuda")
    lib = nat.load()
    nat.check(
        lib.tropnn_b200_trop_code_transpose(
            code.data_ptr(), nat.F16, 37, 8, 96, out.data_ptr(), torch.cuda.current_stream().cuda_stream
        ),
        "trop_code_transpose",
    )
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), code.reshape(37 * 8, 96).t().cpu())


def test_no_device_error_after_tensor_core_runs():
    import ctypes

    _check(items=512, heads=64, cells=16, code_dim=128, dtype=torch.float16, training=True)
    flag = ctypes.c_int(-1)
    nat.check(nat.load().tropnn_b200_device_error(ctypes.byref(flag)), "device_error")
    assert flag.value == 0


@pytest.mark.parametrize(("heads", "cells", "dim"), [(1024, 16, 256), (10, 3, 40), (9, 3, 40), (5, 3, 7)])
def test_code_transpose_exact(heads: int, cells: int, dim: int) -> None:
    """code [H, K, D] -> code^T [D, H*K], bit for bit (the paired-word kernel for even sizes, the
    element kernel otherwise)."""
    lib = nat.load()
    code = torch.randn(heads, cells, dim, device="cuda").half()
    out = torch.empty((dim, heads * cells), device="cuda", dtype=torch.float16)
    nat.check(lib.tropnn_b200_trop_code_transpose(code.data_ptr(), nat.F16, heads, cells, dim, out.data_ptr(),
                                                  nat.stream_handle(code.device)), "trop_code_transpose")
    torch.cuda.synchronize()
    assert torch.equal(out, code.reshape(heads * cells, dim).t())


@pytest.mark.parametrize(("rows", "cols", "src"), [(16384, 256, torch.float32), (16384, 256, torch.float16),
                                                   (301, 64, torch.float32), (2, 5, torch.bfloat16)])
def test_transpose_to_half_exact(rows: int, cols: int, src: torch.dtype) -> None:
    """x [rows, cols] -> half(x)^T [cols, rows] (no gradient scale), bit for bit."""
    lib = nat.load()
    dst = torch.bfloat16 if src == torch.bfloat16 else torch.float16
    x = torch.randn(rows, cols, device="cuda").to(src)
    out = torch.empty((cols, rows), device="cuda", dtype=dst)
    nat.check(lib.tropnn_b200_transpose_to_half(x.data_ptr(), nat.float_code(src), rows, cols, nat.float_code(dst), None,
                                                out.data_ptr(), nat.stream_handle(x.device)), "transpose_to_half")
    torch.cuda.synchronize()
    assert torch.equal(out, x.to(dst).t())


@pytest.mark.parametrize(("rows", "cols", "dtype"), [(302, 6, torch.float16), (3, 7, torch.float16),
                                                     (130, 66, torch.bfloat16)])
def test_transpose_to_half_half_input_shapes(rows: int, cols: int, dtype: torch.dtype) -> None:
    """Half in, half out, no scale (the paired 4-byte transpose, or 2-byte moves for odd shapes):
    a plain transpose, bit for bit."""
    lib = nat.load()
    x = torch.randn(rows, cols, device="cuda").to(dtype)
    out = torch.full((cols, rows), float("nan"), device="cuda", dtype=dtype)
    nat.check(lib.tropnn_b200_transpose_to_half(x.data_ptr(), nat.float_code(dtype), rows, cols, nat.float_code(dtype),
                                                None, out.data_ptr(), nat.stream_handle(x.device)), "transpose_to_half")
    torch.cuda.synchronize()
    assert torch.equal(out, x.t())


@pytest.mark.parametrize(
    ("rows", "cols", "dtype", "scale"),
    [(16384, 256, torch.float16, 1e-6), (2048, 256, torch.float16, None), (302, 68, torch.bfloat16, 1e3),
     (2, 4, torch.float16, None), (130, 132, torch.float16, 1e-3)],
)
def test_split_transpose_half_matches_the_two_passes(rows: int, cols: int, dtype: torch.dtype, scale) -> None:
    """tropnn_b200_split_transpose_half writes split_half's [hi | lo] and transpose_to_half's hi^T
    bit for bit, with and without a gradient scale (tiles of 64 rows x 64 columns: ragged edges in
    both directions)."""
    lib = nat.load()
    stream = nat.stream_handle(torch.device("cuda"))
    code = nat.float_code(dtype)
    gen = torch.Generator().manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=gen) * (1.0 if scale is None else scale)).cuda()
    gmax = None
    if scale is not None:
        gmax = torch.zeros(1, device="cuda", dtype=torch.int32)
        nat.check(lib.tropnn_b200_absmax_f32(x.data_ptr(), x.numel(), gmax.data_ptr(), stream), "absmax")
    want_split = torch.empty((rows, 2 * cols), device="cuda", dtype=dtype)
    want_t = torch.empty((cols, rows), device="cuda", dtype=dtype)
    nat.check(lib.tropnn_b200_split_half(x.data_ptr(), rows, cols, code, nat.ptr(gmax), want_split.data_ptr(), stream),
              "split_half")
    nat.check(lib.tropnn_b200_transpose_to_half(x.data_ptr(), nat.F32, rows, cols, code, nat.ptr(gmax),
                                                want_t.data_ptr(), stream), "transpose_to_half")
    got_split = torch.full((rows, 2 * cols), float("nan"), device="cuda", dtype=dtype)
    got_t = torch.full((cols, rows), float("nan"), device="cuda", dtype=dtype)
    nat.check(lib.tropnn_b200_split_transpose_half(x.data_ptr(), rows, cols, code, nat.ptr(gmax), got_split.data_ptr(),
                                                   got_t.data_ptr(), stream), "split_transpose_half")
    torch.cuda.synchronize()
    assert torch.equal(got_split.view(torch.int16), want_split.view(torch.int16))
    assert torch.equal(got_t.view(torch.int16), want_t.view(torch.int16))


def test_split_transpose_half_rejects_odd_rows() -> None:
    lib = nat.load()
    x = torch.randn(3, 4, device="cuda")
    split = torch.empty((3, 8), device="cuda", dtype=torch.float16)
    xt = torch.empty((4, 3), device="cuda", dtype=torch.float16)
    status = lib.tropnn_b200_split_transpose_half(x.data_ptr(), 3, 4, nat.F16, None, split.data_ptr(), xt.data_ptr(),
                                                  nat.stream_handle(x.device))
    with pytest.raises(ValueError, match="must be even"):
        nat.check(status, "split_transpose_half")


def _split_half(hidden: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    lib = nat.load()
    rows, cols = hidden.shape
    out = torch.empty((rows, 2 * cols), device=hidden.device, dtype=dtype)
    nat.check(lib.tropnn_b200_split_half(hidden.data_ptr(), rows, cols, nat.float_code(dtype), None, out.data_ptr(),
                                         nat.stream_handle(hidden.device)), "split_half")
    return out


@pytest.mark.parametrize(
    ("items", "heads", "cells", "code_dim", "dtype", "training", "use_tc", "workspace"),
    [
        (640, 1024, 16, 256, torch.float16, True, True, True),  # split contraction: slice_reduce writes it
        (640, 1024, 16, 256, torch.bfloat16, False, True, False),  # one CTA per row block: the kernel epilogue
        (20000, 64, 16, 128, torch.float16, False, True, True),  # persistent loop, unsplit
        (300, 12, 16, 64, torch.bfloat16, True, True, True),  # ragged rows
        (300, 12, 16, 64, torch.float16, True, False, False),  # gather path: split_half after it
    ],
)
def test_hidden_split_operand(items, heads, cells, code_dim, dtype, training, use_tc, workspace):
    """The [hi | lo] split written beside hidden equals split_half(hidden) bit for bit, and the
    hidden written with it equals the hidden written without it."""
    gen = torch.Generator().manual_seed(21)
    latent = torch.randn(items, code_dim, generator=gen).to(dtype).cuda()
    code = (torch.randn(heads, cells, code_dim, generator=gen) * 0.5).to(dtype).cuda()
    winner, runner, margins = (t.cuda() for t in _routes(items, heads, cells, gen))
    split = torch.full((items, 2 * code_dim), float("nan"), device="cuda", dtype=dtype)
    with_split = _hidden(latent, code, winner, runner, margins, 0.03, training, use_tc, workspace, split=split)
    plain = _hidden(latent, code, winner, runner, margins, 0.03, training, use_tc, workspace)
    assert np.array_equal(with_split, plain)
    expect = _split_half(torch.from_numpy(with_split).cuda(), dtype)
    torch.cuda.synchronize()
    assert torch.equal(split.view(torch.int16), expect.view(torch.int16))
