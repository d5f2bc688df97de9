"""Throughput of tropnn's routed-layer hot path on B200 (backend="b200").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--secondary NAME]
                    [--impl b200|reference]

Metric: rows/s of TropLinear / PairwiseLinear forward + backward. The
default workload is BASELINE config 5, the configuration the metric is quoted on: the
TropLinear(4096->4096, heads=1024, cells=16, code_dim=256) train step with f16 parameters
(forward, min-face backward of an upstream gradient ~ N(0,1), every parameter gradient)
on a global batch of 16384 rows, split evenly over the N GPUs (strong scaling; at N>1 each
step ends with the all-reduce of the parameter gradients). The config 5
PairwiseLinear(4096->4096, tables=1024, comparisons=8) train step follows as a second keyed
result (``secondary``). Other workloads are selectable with --workload. Data are seeded
synthetic tensors of the configured shapes.

One step = (untimed L2 flush) -> [timed: zero grads, forward, backward, grad
all-reduce]. W warm-up steps, then exactly K timed steps bracketed by barrier +
synchronize, each timed with CUDA events on the launching stream; the max over ranks
is reported. ``e2e`` repeats the step through the same public API with the inputs
copied from pinned host memory and the output + input gradient copied back inside the
timed region, in two forms: a prefetching pipeline (the copies of neighbouring steps
overlap the compute on two copy streams; every step's copies and L2 flush are inside the
timed span) and each step in sequence; ``e2e`` is the faster, ``e2e_modes`` has both.
``roofline`` is the dominant kernel's algorithmic work per launch over its mean
CUDA-event duration in the timed region. ``cpu_baseline`` times the reference's CPU path
(below) on the host cores (rank 0, N=1 only).

``--impl reference`` runs the CPU arm on rank 0 (the other ranks exit without work): the
reference package's own torch CPU path (its default ``backend="torch"``), imported unmodified
from where the reference arm installs it (``baseline/_ref``), on every host core through
torch's threads, on a bounded row sample per step. Without that install it times the numpy
port of the same path (``oracle/``) on all cores as single-threaded processes, and for config
1 eval the C++ restatement of the reference's Zig CPU inference kernels (its faster CPU path
there); ``--cpu-impl`` picks one.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "TropLinear/PairwiseLinear rows/s fwd+bwd, 1-8 B200; % of HBM/TC roofline"
PEAKS_PATH = REPO / "MEASURED_PEAKS.json"
TRAFFIC_PATH = REPO / "profiles" / "traffic.json"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 * 1024 * 1024


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------


@dataclass
class Workload:
    name: str
    kind: str  # "pairwise" | "trop" | "trop_clf" | "pair_clf" (the two-layer classifiers)
    in_features: int
    out_features: int
    rows_per_gpu: int
    train: bool
    dtype: str = "float32"
    layer_kwargs: dict = field(default_factory=dict)
    description: str = ""
    cpu_sample_rows: int = 0  # rows per CPU-baseline step (0 = the full per-GPU batch)
    # The reference's faster CPU path on this workload: "torch" (its default backend) or "zig"
    # (its CPU inference kernels, eval only). Config 1 eval, 8 rows: Zig ~2x the torch path;
    # config 5 eval: the torch path's BLAS scores beat the Zig per-cell dot products.
    cpu_impl: str = "torch"
    hidden: int = 0  # classifiers: width of the hidden layer
    # "weak": rows_per_gpu rows on every rank; "strong": rows_per_gpu is the global batch,
    # split evenly over the ranks (config 5 is quoted on a fixed global batch).
    scaling: str = "weak"

    def rows_on_rank(self, world: int) -> int:
        if self.scaling == "strong":
            if self.rows_per_gpu % world:
                raise SystemExit(f"{self.name}: global batch {self.rows_per_gpu} does not split over {world} ranks")
            return self.rows_per_gpu // world
        return self.rows_per_gpu

    def global_rows(self, world: int) -> int:
        return self.rows_per_gpu if self.scaling == "strong" else self.rows_per_gpu * world

    # rows per step when the reference package's own torch path is timed (one process on every
    # host core); 0 = the numpy-port sample size.
    ref_sample_rows: int = 0

    @property
    def cpu_rows(self) -> int:
        return self.cpu_sample_rows or self.rows_per_gpu

    @property
    def ref_rows(self) -> int:
        return self.ref_sample_rows or self.cpu_rows

    @property
    def classifier(self) -> bool:
        return self.kind in ("trop_clf", "pair_clf")

    def build(self):
        import tropnn_b200

        if self.classifier:
            # examples/emnist.py:121-175: routed layers in_features -> hidden -> out_features,
            # seeds seed + index, no activation between them.
            cls = tropnn_b200.TropLinear if self.kind == "trop_clf" else tropnn_b200.PairwiseLinear
            dims = [self.in_features, self.hidden, self.out_features]
            return _Classifier([cls(a, b, seed=i, **self.layer_kwargs) for i, (a, b) in enumerate(zip(dims[:-1], dims[1:]))])
        cls = tropnn_b200.PairwiseLinear if self.kind == "pairwise" else tropnn_b200.TropLinear
        layer = cls(self.in_features, self.out_features, seed=0, **self.layer_kwargs)
        if self.dtype == "float16":
            layer = layer.half()
        return layer


class _Classifier(torch.nn.Module):
    """The reference example's routed classifier (examples/emnist.py:121-175): 2-D input lifted
    to one step, the routed layers applied in order, the step axis dropped again."""

    def __init__(self, layers: list) -> None:
        super().__init__()
        self.layers = torch.nn.ModuleList(layers)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.ndim == 2:
            x = x.unsqueeze(1)
        for layer in self.layers:
            x = layer(x)
        return x.squeeze(1)


WORKLOADS = {
    "pairwise_cfg2": Workload(
        "pairwise_cfg2", "pairwise", 256, 512, 4096, True,
        layer_kwargs=dict(tables=16, comparisons=6, surrogate="fast_sigmoid_odd", use_min_margin_ste=True),
        description="BASELINE config 2: PairwiseLinear(256->512, tables=16, comparisons=6), fp32, fwd + STE bwd, batch 4096",
    ),
    "pairwise_cfg2_b8": Workload(
        "pairwise_cfg2_b8", "pairwise", 256, 512, 8, True,
        layer_kwargs=dict(tables=16, comparisons=6, surrogate="fast_sigmoid_odd", use_min_margin_ste=True),
        description="BASELINE config 2 at batch 8: PairwiseLinear(256->512, tables=16, comparisons=6), fp32, fwd + STE bwd",
    ),
    "trop_cfg3_clf": Workload(
        "trop_cfg3_clf", "trop_clf", 784, 10, 512, True, hidden=128,
        layer_kwargs=dict(heads=256, cells=16, code_dim=64),
        description="BASELINE config 3: TropLinear classifier 784->128->10 (H256, K16, D64), fp32, one train step "
        "(fwd, cross-entropy, min-face bwd, Adam lr 1e-3), batch 512, x ~ U[0,1], labels ~ U{0..9}",
    ),
    "pair_cfg4_clf": Workload(
        "pair_cfg4_clf", "pair_clf", 784, 10, 512, True, hidden=128,
        layer_kwargs=dict(tables=136, comparisons=6),
        description="BASELINE config 4: PairwiseLinear classifier 784->128->10 (T136, C6), fp32, one train step "
        "(fwd, cross-entropy, STE/LUT-grad bwd, Adam lr 1e-3), batch 512, x ~ U[0,1], labels ~ U{0..9}",
    ),
    "trop_cfg1": Workload(
        "trop_cfg1", "trop", 256, 512, 8, False,
        layer_kwargs=dict(heads=32, cells=4, code_dim=32),
        description="BASELINE config 1: TropLinear(256->512, H32, K4, D32), fp32, eval forward, batch 8",
        cpu_impl="zig",
    ),
    "trop_cfg3_layer1": Workload(
        "trop_cfg3_layer1", "trop", 784, 128, 512, True,
        layer_kwargs=dict(heads=256, cells=16, code_dim=64),
        description="config 3 layer 1: TropLinear(784->128, H256, K16, D64), fp32, fwd + min-face bwd, batch 512",
    ),
    "pairwise_cfg5_train": Workload(
        "pairwise_cfg5_train", "pairwise", 4096, 4096, 16384, True, dtype="float16",
        layer_kwargs=dict(tables=1024, comparisons=8),
        description="config 5: PairwiseLinear(4096->4096, T1024, C8), f16 params, train step, batch 16384",
        cpu_sample_rows=64,
        scaling="strong",
        ref_sample_rows=2,
    ),
    "trop_cfg5_eval": Workload(
        "trop_cfg5_eval", "trop", 4096, 4096, 65536, False, dtype="float16",
        layer_kwargs=dict(heads=1024, cells=16, code_dim=256),
        description="config 5: TropLinear(4096->4096, H1024, K16, D256), f16 params, eval forward, batch 65536",
        cpu_sample_rows=256,
        scaling="strong",
        ref_sample_rows=64,
    ),
    "pairwise_cfg5_eval": Workload(
        "pairwise_cfg5_eval", "pairwise", 4096, 4096, 65536, False, dtype="float16",
        layer_kwargs=dict(tables=1024, comparisons=8),
        description="config 5: PairwiseLinear(4096->4096, T1024, C8), f16 params, eval forward, batch 65536",
        cpu_sample_rows=32,
        scaling="strong",
        ref_sample_rows=4,
    ),
    "trop_cfg5_train": Workload(
        "trop_cfg5_train", "trop", 4096, 4096, 16384, True, dtype="float16",
        layer_kwargs=dict(heads=1024, cells=16, code_dim=256),
        description="config 5: TropLinear(4096->4096, H1024, K16, D256), f16 params, train step (fwd + min-face bwd), batch 16384",
        cpu_sample_rows=32,
        scaling="strong",
        ref_sample_rows=16,
    ),
}


# A table at most this large stays in the 126 MB L2 across a launch: its gathered rows are L2
# hits, and only its first read reaches HBM.
L2_RESIDENT_BYTES = 64 << 20


def lut_l2_resident(w: Workload) -> bool:
    """Whether a Pairwise workload's LUT fits the L2 share that keeps its gathers off HBM."""
    kw = w.layer_kwargs
    elt = 2 if w.dtype == "float16" else 4
    return w.kind == "pairwise" and kw["tables"] * (1 << kw["comparisons"]) * w.out_features * elt <= L2_RESIDENT_BYTES


def algorithmic_bytes(w: Workload, kernel: str, rows: int) -> float | None:
    """Algorithmic bytes one launch of ``kernel`` moves for ``rows`` rows (per-row formulas of
    the hot-path measurement plan; parameter bytes counted once per gathered row). An
    L2-resident Pairwise LUT (config 2) is counted once per launch instead: its per-row gathers
    never reach HBM, so counting them would put the HBM fraction above 1."""
    if w.classifier:
        return None  # two layers of different shapes share the kernel names
    kw = w.layer_kwargs
    elt = 2 if w.dtype == "float16" else 4
    if w.kind == "pairwise":
        T, C, out, inn = kw["tables"], kw["comparisons"], w.out_features, w.in_features
        lut_bytes = T * (1 << C) * out * elt
        resident = lut_l2_resident(w)
        gathered = 0 if resident else 1
        per_row = {
            "pairwise_forward": gathered * T * out * elt + inn * 4 + out * 4 + T * 8 + T * C * 4,
            "pairwise_ste_backward": out * 4 + gathered * 2 * T * out * elt + inn * 4 + T * 8 + T * C * 4 + T * 4 + T,
            "pairwise_lut_grad": T * out * 4 + T * 4,
            "bucket_sort": T * 8 + T * 4,
            "pairwise_threshold_grad": T * 4 + T,
        }.get(kernel)
        if per_row is None:
            return None
        once = kernel == "pairwise_lut_grad" or (resident and kernel in ("pairwise_forward", "pairwise_ste_backward"))
        return float(per_row * rows + (lut_bytes if once else 0))
    H, K, D = kw["heads"], kw["cells"], kw["code_dim"]
    per_row = {
        "trop_route": D * 4 + H * (8 + 1 + 1 + 4),
        "trop_hidden": H * D * elt * (2 if w.train else 1) + 2 * D * 4 + H * (2 + 4),
        "trop_backward_rows": 4 * H * D * elt + 2 * D * 4 + H * (2 + 4 + 12),
        "trop_code_grad": 2 * D * 4 + 2 * 8,
        "trop_router_grad": 2 * D * 4 + 2 * 8,
        "bucket_sort": H * (1 + 4),
    }.get(kernel)
    if per_row is None:
        return None
    fixed = H * K * D * elt if kernel in ("trop_code_grad", "trop_router_grad") else 0
    return float(per_row * rows + fixed)


def tensor_core_route(w: Workload, rows: int) -> bool:
    """Whether trop_route runs on the tcgen05 tensor cores for this workload (the C ABI's rule:
    kind::f16 for half parameters, 3xTF32 for f32 parameters with code_dim <= 128 from 64 rows on)."""
    if w.kind != "trop":
        return False
    kw = w.layer_kwargs
    H, K, D = kw["heads"], kw["cells"], kw["code_dim"]
    if w.dtype == "float32":
        return K in (2, 4, 8, 16, 32) and D % 4 == 0 and D <= 128 and H * K >= 32 and rows >= 64
    return K in (2, 4, 8, 16, 32) and D % 8 == 0 and (D + 63) // 64 <= 8 and rows >= 128 and H * K >= 128


def tensor_core_hidden(w: Workload, rows: int) -> bool:
    """Whether the code sum runs as the one-hot tcgen05 GEMM (the C ABI's rule)."""
    if w.kind != "trop" or w.dtype == "float32":
        return False
    kw = w.layer_kwargs
    H, K, D = kw["heads"], kw["cells"], kw["code_dim"]
    return K in (2, 4, 8, 16, 32) and D % 64 == 0 and 64 <= D <= 256 and (H * K) % 8 == 0 and rows >= 128


def kernel_roofline(w: Workload, kernel: str, rows: int, peaks: dict) -> tuple[str, float, str, float, str] | None:
    """(bound, work per launch, unit, peak, peak label) of one kernel: executed FLOPs against
    the measured bf16 tensor peak for the f16/bf16 tcgen05 GEMMs (route scores, one-hot code
    sum, the output map when its FLOPs outweigh its f32 output bytes, the min-face backward
    GEMMs), against half that peak for the tf32 output-map gradients (kind::tf32 runs at half
    the f16 rate), bytes against the measured HBM copy bandwidth for everything else."""
    tc_peak, hbm_peak = peaks["bf16_tflops"], peaks["hbm_gbs"]
    tc, tf32, hbm = (tc_peak, "bf16_tflops"), (tc_peak / 2, "bf16_tflops / 2 (tf32)"), (hbm_peak, "hbm_gbs")
    if w.kind == "trop":
        kw = w.layer_kwargs
        H, K, D, out = kw["heads"], kw["cells"], kw["code_dim"], w.out_features
        hk = H * K
        if kernel == "trop_route" and tensor_core_route(w, rows):
            # f32 parameters run kind::tf32 (half the f16 rate) with three products per step.
            if w.dtype == "float32":
                return "tensor", 3 * 2.0 * hk * D * rows, "TFLOP/s", *tf32
            return "tensor", 2.0 * hk * D * rows, "TFLOP/s", *tc
        if kernel == "trop_proj":
            # z = half(x) P^T: 2 in D FLOP a row; x read once in f32 (in * 4 bytes a row): the
            # slower of the two bounds.
            inn = w.in_features
            flops = 2.0 * rows * inn * D
            nbytes = float(rows * inn * 4 + rows * D * 2 + D * inn * 2)
            if flops / (tc_peak * 1e12) >= nbytes / (hbm_peak * 1e9):
                return "tensor", flops, "TFLOP/s", *tc
            return "hbm", nbytes, "GB/s", *hbm
        if kernel == "trop_proj_wgrad":
            # grad_P = g^T half(x): x read once in f32, g^T [D, rows] and grad_P once in half.
            inn = w.in_features
            return "hbm", float(rows * inn * 4 + D * rows * 2 + D * inn * 2), "GB/s", *hbm
        if kernel == "trop_hidden" and tensor_core_hidden(w, rows):
            return "tensor", 2.0 * hk * D * rows, "TFLOP/s", *tc
        if kernel == "linear_f32out":
            flops = 2.0 * rows * out * 2 * D  # [hi | lo] slices against one weight
            nbytes = float(rows * out * 4 + rows * 2 * D * 2 + out * D * 2 + out * 4)
            if flops / (tc_peak * 1e12) >= nbytes / (hbm_peak * 1e9):
                return "tensor", flops, "TFLOP/s", *tc
            return "hbm", nbytes, "GB/s", *hbm
        if kernel == "trop_gm":  # [hi | lo] g against the code table, route-picking epilogue
            return "tensor", 2.0 * rows * hk * 2 * D, "TFLOP/s", *tc
        if kernel in ("trop_router_term", "trop_code_grad", "trop_router_grad"):
            return "tensor", 2.0 * rows * hk * D, "TFLOP/s", *tc
        if kernel == "linear_dgrad":  # big and small g against the weight
            return "tensor", 2.0 * 2 * rows * out * D, "TFLOP/s", *tf32
        if kernel == "linear_wgrad":  # big*big, small*big, big*small
            return "tensor", 2.0 * 3 * rows * out * D, "TFLOP/s", *tf32
        if kernel == "split_half":
            return "hbm", float(rows * D * 4 + rows * 2 * D * 2), "GB/s", *hbm
        if kernel == "split_transpose_half":  # f32 g in, [hi | lo] and hi^T out
            return "hbm", float(rows * D * (4 + 4 + 2)), "GB/s", *hbm
        if kernel == "tf32_split":
            return "hbm", float(rows * D * 12), "GB/s", *hbm
        if kernel == "transpose_to_half":
            return "hbm", float(rows * D * (4 + 2)), "GB/s", *hbm
        if kernel == "trop_code_transpose":
            return "hbm", float(2 * hk * D * 2), "GB/s", *hbm
    work = algorithmic_bytes(w, kernel, rows)
    if work is None:
        return None
    return "hbm", work, "GB/s", *hbm


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def _peaks() -> tuple[dict, str]:
    if PEAKS_PATH.exists():
        return json.loads(PEAKS_PATH.read_text()), "measured"
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS}, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, device: torch.device) -> None:
        # nvidia-smi numbers GPUs independently of CUDA_VISIBLE_DEVICES; select by UUID.
        self.device_index = f"GPU-{torch.cuda.get_device_properties(device).uuid}"
        self.proc: subprocess.Popen | None = None
        self.lines: list[str] = []
        self._thread: threading.Thread | None = None

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
            time.sleep(0.3)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            with contextlib.suppress(Exception):
                self.proc.wait(timeout=5)
            if self._thread is not None:
                self._thread.join(timeout=2)

    def summary(self) -> dict:
        mhz: list[float] = []
        max_mhz: list[float] = []
        reasons: set[str] = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz.append(float(parts[2]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower() == "active":
                    reasons.add(name)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {
            "sm_mhz": statistics.median(mhz),
            "sm_max_mhz": max(max_mhz),
            "reasons": sorted(reasons),
            "samples": len(mhz),
        }


def _dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def _max_over_ranks(value: float, world: int, device: torch.device) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier_sync(world: int, device: torch.device) -> None:
    torch.cuda.synchronize(device)
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


# ---------------------------------------------------------------------------
# b200 arm
# ---------------------------------------------------------------------------


def _make_inputs(w: Workload, rank: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """x and the upstream gradient, or for the classifiers x ~ U[0,1] and labels ~ U{0..C-1}."""
    gen = torch.Generator().manual_seed(1 + rank)
    if w.classifier:
        x = torch.rand(w.rows_per_gpu, w.in_features, generator=gen)
        labels = torch.randint(0, w.out_features, (w.rows_per_gpu,), generator=gen)
        return x, labels
    x = torch.randn(w.rows_per_gpu, w.in_features, generator=gen)
    g = torch.randn(w.rows_per_gpu, 1, w.out_features, generator=gen)
    return x, g


def _input_grad(w: Workload) -> bool:
    """Whether the step wants d(loss)/dx (the layer workloads' upstream-gradient steps)."""
    return w.train and not w.classifier


def _step(layer, x: torch.Tensor, g: torch.Tensor | None, w: Workload) -> torch.Tensor:
    """One forward (+ backward) of the layer through its public module API. Classifiers: the
    logits' cross-entropy against the labels ``g``, backward, the loss returned (the optimizer
    step follows the gradient all-reduce: ``_optimizer_step``)."""
    if w.classifier:
        layer.optimizer.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(layer(x), g)
        loss.backward()
        return loss
    if w.train:
        for p in layer.parameters():
            p.grad = None
        x.grad = None  # the input's gradient is the step's output, not an accumulator
        y = layer(x)
        y.backward(g)
        return y
    with torch.no_grad():
        return layer(x)


def _optimizer_step(layer) -> None:
    opt = getattr(layer, "optimizer", None)
    if opt is not None:
        opt.step()


def _results(w: Workload, y: torch.Tensor, xd: torch.Tensor) -> list[torch.Tensor]:
    """Device tensors a step hands back to the host: the loss (classifiers), or the output and,
    when training, the input gradient."""
    if w.classifier:
        return [y.detach().reshape(1)]
    out = [y.detach().float()]
    if w.train:
        out.append(xd.grad)
    return out


def _result_buffers(w: Workload, x_host: torch.Tensor) -> list[torch.Tensor]:
    """Pinned host buffers matching ``_results``."""
    if w.classifier:
        return [torch.empty(1, dtype=torch.float32).pin_memory()]
    bufs = [torch.empty((w.rows_per_gpu, 1, w.out_features), dtype=torch.float32).pin_memory()]
    if w.train:
        bufs.append(torch.empty_like(x_host).pin_memory())
    return bufs


def _capture(fn, device: torch.device, during_capture=contextlib.nullcontext) -> torch.cuda.CUDAGraph:
    """Captures ``fn`` (warmed up on a side stream first) into a CUDA graph."""
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with during_capture(), torch.cuda.graph(graph):
        fn()
    torch.cuda.synchronize(device)
    return graph


def _timed(steps: int, body, flush: torch.Tensor, world: int, device: torch.device) -> float:
    """Sum of per-step CUDA-event durations (ms) of ``steps`` calls of ``body``, with an
    untimed L2 flush before each step; barrier + synchronize on both sides."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    _barrier_sync(world, device)
    for i in range(steps):
        flush.fill_(float(i))
        starts[i].record()
        body()
        ends[i].record()
    _barrier_sync(world, device)
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends))


def _pipelined_e2e(steps, layer, w, x_pin, g_pin, out_pins, reduce_grads, flush, world, device) -> float:
    """``steps`` e2e steps as a prefetching pipeline; returns the device time (ms) of the whole
    span, from before the first input copy to after the last result copy.

    Step i: the copy-in stream uploads the pinned inputs into device buffer i % 2 (once step
    i-2 has finished with it); the compute stream flushes L2 and runs the step through the
    module API; the copy-out stream copies the step's results (``_results``) into pinned
    buffer set i % 2. Events order the three streams, and ``record_stream`` keeps the step's
    output tensors alive until their copy has run."""
    if steps == 0:
        return 0.0
    comp = torch.cuda.current_stream(device)
    cin, cout = torch.cuda.Stream(device), torch.cuda.Stream(device)
    xd = [torch.empty(x_pin.shape, dtype=x_pin.dtype, device=device) for _ in range(2)]
    gd = [torch.empty(g_pin.shape, dtype=g_pin.dtype, device=device) for _ in range(2)] if w.train else [None, None]
    out_host = [out_pins, [torch.empty_like(b).pin_memory() for b in out_pins]]
    in_ready = [torch.cuda.Event() for _ in range(steps)]
    done = [torch.cuda.Event() for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def upload(i: int) -> None:
        with torch.cuda.stream(cin):
            if i >= 2:
                cin.wait_event(done[i - 2])
            xd[i % 2].copy_(x_pin, non_blocking=True)
            if w.train:
                gd[i % 2].copy_(g_pin, non_blocking=True)
            in_ready[i].record(cin)

    _barrier_sync(world, device)
    start.record(comp)
    cin.wait_event(start)
    upload(0)
    for i in range(steps):
        if i + 1 < steps:
            upload(i + 1)
        comp.wait_event(in_ready[i])
        flush.fill_(float(i))
        xi = xd[i % 2].detach().requires_grad_(_input_grad(w))
        y = _step(layer, xi, gd[i % 2], w)
        reduce_grads()
        done[i].record(comp)
        with torch.cuda.stream(cout):
            cout.wait_event(done[i])
            for buf, r in zip(out_host[i % 2], _results(w, y, xi)):
                r.record_stream(cout)
                buf.copy_(r, non_blocking=True)
    comp.wait_stream(cout)
    comp.wait_stream(cin)
    end.record(comp)
    _barrier_sync(world, device)
    return start.elapsed_time(end)


def _init_dist(device: torch.device, world: int) -> None:
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))


def _end_dist(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_b200(args: argparse.Namespace, w: Workload) -> dict | None:
    """One workload on this rank's GPU (process group already set up at N>1); rank 0 gets the
    JSON line's fields, the other ranks None."""
    import dataclasses

    import tropnn_b200
    from tropnn_b200.distributed import PeerAllReduce, fused_lut_allreduce

    rank, world, local_rank = _dist_env()
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    tropnn_b200._native.load()
    # This rank's share of the step: the whole per-GPU batch (weak scaling) or an even slice
    # of the global batch (strong scaling).
    w_rank = dataclasses.replace(w, rows_per_gpu=w.rows_on_rank(world), scaling="weak")
    layer = w_rank.build().to(device).train(w.train)
    if w.classifier:
        # Adam as the reference example trains (examples/emnist.py:310, AdamW with weight_decay 0),
        # capturable so that the whole step goes into one CUDA graph.
        layer.optimizer = torch.optim.Adam(layer.parameters(), lr=1e-3, capturable=True)
    peer = peer_lut = None
    with contextlib.ExitStack() as stack:
        if world > 1 and w.train:
            grads = [p for p in layer.parameters() if p.requires_grad]
            numel = sum(p.numel() for p in grads)
            # auto: the peer kernel where it was measured faster than NCCL (2 and 4 GPUs).
            use_peer = {"auto": world <= 4, "peer": world <= PeerAllReduce.max_ranks(), "nccl": False}[args.allreduce]
            if use_peer and all(p.dtype == torch.float32 for p in grads) and numel <= 1 << 24:
                # f32 gradients of a few MiB: the NVLink peer-memory all-reduce kernel
                # (one-shot; NCCL's protocol is latency-bound at this size on two GPUs).
                peer = PeerAllReduce(numel)
                if w.kind == "pairwise" and args.fuse_lut_allreduce:
                    # The LUT gradient's average runs inside the LUT-gradient kernel (a peer
                    # set of its own); the rest goes through `peer` after the backward.
                    kw = w.layer_kwargs
                    cap = PeerAllReduce.lut_capacity(kw["tables"], kw["comparisons"], w.out_features)
                    if cap > 0:
                        peer_lut = PeerAllReduce(cap)
                        stack.enter_context(fused_lut_allreduce(peer_lut))
        try:
            return _run_b200_body(args, w, w_rank, rank, world, device, layer, peer)
        finally:
            stack.close()
            if peer_lut is not None:
                peer_lut.close()
            if peer is not None:
                peer.close()
            del layer
            torch.cuda.synchronize(device)
            torch.cuda.empty_cache()


def _run_b200_body(
    args: argparse.Namespace, w: Workload, w_rank: Workload, rank: int, world: int, device: torch.device, layer, peer
) -> dict | None:
    from tropnn_b200 import _native as nat
    from tropnn_b200 import trace
    from tropnn_b200.distributed import allreduce_gradients, fused_lut_peer

    x_host, g_host = _make_inputs(w_rank, rank, device)
    x = x_host.to(device).requires_grad_(_input_grad(w))
    g = g_host.to(device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def reduce_grads() -> None:
        """After the backward: the gradient all-reduce at N>1, then the optimizer step
        (classifiers)."""
        if world > 1 and w.train:
            allreduce_gradients(layer, peer=peer)
        _optimizer_step(layer)

    def eager_step() -> None:
        _step(layer, x, g, w)
        reduce_grads()

    for _ in range(args.warmup):
        eager_step()
    _barrier_sync(world, device)

    # Timed region: the step, with the gradient all-reduce at N>1, captured once as a
    # CUDA graph (no host launch gaps) and replayed.
    def full_step() -> None:
        _step(layer, x, g, w)
        reduce_grads()

    graph = _capture(full_step, device)
    sampler = ClockSampler(device)

    def graph_step() -> None:
        graph.replay()

    with sampler:
        total_ms = _max_over_ranks(_timed(args.steps, graph_step, flush, world, device), world, device)

    # Per-kernel device time: a second capture with CUDA events around every b200 launch.
    holder: dict = {}

    @contextlib.contextmanager
    def tracing():
        lib = nat.load()
        before = lib.tropnn_b200_kernel_launches()
        with trace.launch_trace() as t:
            holder["trace"] = t
            yield
        # The library's own count of the kernels the captured step launches (an entry point
        # can launch several: split-contraction reductions, the staged kernels' waves).
        holder["kernels"] = lib.tropnn_b200_kernel_launches() - before

    traced = _capture(lambda: _step(layer, x, g, w), device, during_capture=tracing)
    tr = holder["trace"]
    launches_per_step = holder["kernels"]
    for i in range(args.steps):
        flush.fill_(float(i))
        traced.replay()
        tr.harvest()
    kernels = tr.summary()
    del traced

    # The same step run eagerly through the module API (host launch overhead included).
    eager_ms = _max_over_ranks(_timed(args.steps, eager_step, flush, world, device), world, device)

    # End to end: eager public API, inputs copied from pinned host memory and the output
    # (+ input gradient) copied back inside the timed region.
    x_pin = x_host.pin_memory()
    g_pin = g_host.pin_memory()
    out_pins = _result_buffers(w_rank, x_host)
    h2d = x_pin.numel() * x_pin.element_size() + (g_pin.numel() * g_pin.element_size() if w.train else 0)
    d2h = sum(b.numel() * b.element_size() for b in out_pins)

    def e2e_step() -> None:
        xd = x_pin.to(device, non_blocking=True).requires_grad_(_input_grad(w))
        gd = g_pin.to(device, non_blocking=True) if w.train else None
        y = _step(layer, xd, gd, w)
        reduce_grads()
        for buf, r in zip(out_pins, _results(w, y, xd)):
            buf.copy_(r, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_serial_ms = _max_over_ranks(_timed(args.steps, e2e_step, flush, world, device), world, device)

    # The same steps as a prefetching pipeline: step i+1's inputs go up on one copy stream
    # and step i-1's results come back on another while step i computes.
    def e2e_pipelined(steps: int) -> float:
        return _pipelined_e2e(steps, layer, w, x_pin, g_pin, out_pins, reduce_grads, flush, world, device)

    e2e_pipelined(args.warmup)
    e2e_ms = _max_over_ranks(e2e_pipelined(args.steps), world, device)
    del graph

    if rank != 0:
        return None

    rows_total = w.global_rows(world)
    value = rows_total * args.steps / (total_ms / 1e3)
    # e2e: the faster of the two end-to-end modes (the pipeline wins when the host copies
    # dominate, the serial form when host launch work does).
    e2e_modes = {"pipelined": e2e_ms, "serial": e2e_serial_ms}
    e2e_mode = min(e2e_modes, key=e2e_modes.get)
    e2e_value = rows_total * args.steps / (e2e_modes[e2e_mode] / 1e3)

    peaks, peaks_kind = _peaks()
    # The captures in profiles/traffic.json are of one GPU running the workload's full batch: at
    # other per-GPU row counts (N > 1, --rows) the launch moves other bytes, so none is attached.
    traffic_table = (
        json.loads(TRAFFIC_PATH.read_text()).get(w.name, {})
        if TRAFFIC_PATH.exists() and world == 1 and not args.rows
        else {}
    )
    per_kernel_roofline = {}
    for name, stats in kernels.items():
        rl = kernel_roofline(w, name, w_rank.rows_per_gpu, peaks)
        if rl is None:
            continue
        bound, work, unit, peak, peak_label = rl
        mean_s = stats["mean_ms"] / 1e3
        achieved = work / mean_s / (1e12 if bound == "tensor" else 1e9)
        traffic = traffic_table.get(name)
        per_kernel_roofline[name] = {
            "kernel": name,
            "bound": bound,
            "achieved": round(achieved, 1),
            "peak": round(peak, 1),
            "peak_source": f"{peaks_kind} {peak_label}",
            "unit": unit,
            "frac": round(achieved / peak, 3),
            "traffic": traffic.get("bytes") if isinstance(traffic, dict) else traffic,
            ("algorithmic_flops_per_launch" if bound == "tensor" else "algorithmic_bytes_per_launch"): work,
            "mean_launch_us": round(mean_s * 1e6, 2),
        }
        if w.kind == "pairwise" and name in ("pairwise_forward", "pairwise_ste_backward"):
            per_kernel_roofline[name]["lut"] = (
                "L2-resident: counted once per launch" if lut_l2_resident(w) else "gathered rows counted per row (logical)"
            )
        if isinstance(traffic, dict):
            # ncu figures of one capture of the same kernel (profiles/): L2 throughput and the
            # DRAM bytes behind a logical-bytes fraction above 1 (L2-resident tables).
            per_kernel_roofline[name]["ncu"] = {k: v for k, v in traffic.items() if k != "bytes"}
    roofline = None
    if per_kernel_roofline:
        top = max(per_kernel_roofline, key=lambda k: kernels[k]["total_ms"])
        roofline = per_kernel_roofline[top]
    step_kernel_ms = sum(v["total_ms"] for v in kernels.values()) / args.steps

    return {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": w.scaling,
        "vs_baseline": None,
        "dtype": "f32" if w.dtype == "float32" else "f16 params / f32 accumulate",
        "data": "synthetic (seeded N(0,1) inputs and upstream grads; seeded default init)",
        "config": {
            "workload": w.description,
            "rows_per_gpu": w_rank.rows_per_gpu,
            "global_batch": rows_total,
            "parallelism": (
                f"dp{world} (batch-row shards, {'NVLink peer-memory' if peer is not None else 'NCCL'} grad all-reduce"
                + (", LUT-gradient average fused into its kernel" if fused_lut_peer() is not None else "")
                + ")"
                if world > 1
                else "single GPU"
            ),
            "l2": f"flushed between timed steps ({L2_FLUSH_BYTES >> 20} MiB write, untimed)",
            "timing": "step (with the gradient all-reduce at N>1) captured as one CUDA graph and replayed",
        },
        "eager": {"value": round(rows_total * args.steps / (eager_ms / 1e3), 1), "unit": "rows/s",
                  "ms_per_step": round(eager_ms / args.steps, 4)},
        "e2e": {
            "value": round(e2e_value, 1),
            "unit": "rows/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "ms_per_step": round(e2e_modes[e2e_mode] / args.steps, 4),
            "mode": e2e_mode,
            "path": (
                ("eager module API, pinned x and labels in, loss out" if w.classifier
                 else "eager module API, pinned host inputs in, output + input gradient out")
                + ("; copies of neighbouring steps overlap the compute on two copy streams; L2 flush per step "
                   "inside the span" if e2e_mode == "pipelined"
                   else "; each step's copies and compute in sequence (untimed L2 flush between steps)")
                + "; the faster of the pipelined and serial modes (both below)"
            ),
        },
        "e2e_modes": {k: {"value": round(rows_total * args.steps / (v / 1e3), 1), "unit": "rows/s",
                          "ms_per_step": round(v / args.steps, 4)} for k, v in e2e_modes.items()},
        "gpu_launches": launches_per_step * args.steps,
        "kernels": {k: {"launches_per_step": v["launches"] // args.steps, "mean_us": round(v["mean_ms"] * 1e3, 2)}
                    for k, v in kernels.items()},
        "kernel_ms_per_step": round(step_kernel_ms, 4),
        "roofline": roofline,
        "kernel_rooflines": {k: {kk: v[kk] for kk in ("bound", "achieved", "unit", "frac")} for k, v in per_kernel_roofline.items()},
        "clocks": sampler.summary(),
    }


# ---------------------------------------------------------------------------
# CPU arm (oracle port of the reference's torch path)
# ---------------------------------------------------------------------------


def _oracle_params(w: Workload, impl: str = "torch") -> tuple[dict[str, np.ndarray], object]:
    """Seeded parameters as numpy. For the torch path half tensors are upcast once (exactly, as
    the reference's ``.to(compute_dtype)`` does on every call) so the timed steps do not repeat
    it; the Zig path reads f16 parameters as they are (its f16 kernels widen per element)."""
    layer = w.build()
    params = {}
    for k, v in layer.state_dict().items():
        a = v.detach().numpy()
        params[k] = a.astype(np.float32) if a.dtype == np.float16 and impl == "torch" else a
    return params, layer


def _classifier_state(w: Workload) -> dict:
    """CPU state of a classifier step: per layer its f32 parameters (numpy), the module (for its
    settings and parameter names) and Adam moments."""
    model = w.build()
    layers = []
    for mod in model.layers:
        params = {k: (v.detach().numpy().astype(np.float32) if v.is_floating_point() else v.detach().numpy())
                  for k, v in mod.state_dict().items()}
        names = [k for k, _ in mod.named_parameters()]
        adam = {k: (np.zeros_like(params[k]), np.zeros_like(params[k])) for k in names}
        layers.append({"module": mod, "params": params, "names": names, "adam": adam})
    return {"layers": layers, "t": 0}


def _adam_update(p: np.ndarray, g: np.ndarray, m: np.ndarray, v: np.ndarray, t: int, lr: float = 1e-3,
                 b1: float = 0.9, b2: float = 0.999, eps: float = 1e-8) -> None:
    """torch.optim.Adam's update (weight_decay 0), in place, float32."""
    f = np.float32
    m *= f(b1)
    m += f(1 - b1) * g
    v *= f(b2)
    v += f(1 - b2) * g * g
    denom = np.sqrt(v) / f(math.sqrt(1 - b2 ** t)) + f(eps)
    p -= f(lr / (1 - b1 ** t)) * m / denom


def _oracle_classifier_step(w: Workload, state: dict, x: np.ndarray, labels: np.ndarray) -> None:
    """One classifier train step in numpy (the reference's torch path): each layer's forward,
    cross-entropy on the logits, each layer's backward in reverse, Adam on every parameter."""
    import oracle

    acts, fwds = [x], []
    for lay in state["layers"]:
        mod, params = lay["module"], lay["params"]
        if w.kind == "trop_clf":
            f = oracle.trop_linear_forward(acts[-1], params, code_scale=mod.code_scale, training=True)
            acts.append(f["y"])
        else:
            f = oracle.pairwise_forward(acts[-1], params["anchors"], params["thresholds"], params["lut"],
                                        output_scale=mod.output_scale)
            acts.append(f["out"])
        fwds.append(f)
    logits = acts[-1].astype(np.float32)
    e = np.exp(logits - logits.max(axis=1, keepdims=True))
    grad = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
    grad[np.arange(len(labels)), labels] -= np.float32(1.0)
    grad /= np.float32(len(labels))
    state["t"] += 1
    for i in reversed(range(len(state["layers"]))):
        lay = state["layers"][i]
        mod, params = lay["module"], lay["params"]
        if w.kind == "trop_clf":
            grads = oracle.trop_linear_backward(grad, acts[i], params, fwds[i], code_scale=mod.code_scale, training=True)
        else:
            grads = oracle.pairwise_backward(
                grad, fwds[i]["indices"], fwds[i]["margins"], params["anchors"], params["lut"], in_features=mod.in_features,
                output_scale=mod.output_scale, use_min_margin_ste=mod.use_min_margin_ste, surrogate=mod.surrogate,
            )
        grad = grads["x"]
        for name in lay["names"]:
            m, v = lay["adam"][name]
            _adam_update(params[name], grads[name], m, v, state["t"])


def _zig_port_usable() -> str | None:
    """None when the C++ Zig restatement builds and loads on this host, else why not."""
    try:
        from oracle import native

        native.build()
        native.load()
    except (OSError, RuntimeError, subprocess.CalledProcessError) as exc:
        return str(exc).splitlines()[0]
    return None


def reference_package_root() -> Path | None:
    """Directory holding the reference package ``tropnn`` as installed for the reference arm
    (``pip install --no-deps --target baseline/_ref <reference source>``), or the directory named
    by ``TROPNN_REFERENCE``; None when neither has it."""
    for root in (os.environ.get("TROPNN_REFERENCE"), str(REPO / "baseline" / "_ref")):
        if root and (Path(root) / "tropnn" / "__init__.py").is_file():
            return Path(root)
    return None


def cpu_impl_for(w: Workload, requested: str) -> str:
    """The CPU path a leg times. "auto": the reference's faster CPU path on the workload: its own
    torch path imported from the installed reference package ("reference") when present, else
    the numpy port of it ("torch"), and for config 1 eval the C++ restatement of its Zig CPU
    inference kernels ("zig", eval workloads only)."""
    if requested == "zig" and w.train:
        raise SystemExit(f"--cpu-impl zig: {w.name} is a training workload; the Zig kernels are inference only")
    if requested == "reference" and reference_package_root() is None:
        raise SystemExit("--cpu-impl reference: the reference package is not installed under baseline/_ref")
    if requested != "auto":
        return requested
    if not w.train and w.cpu_impl == "zig":
        why = _zig_port_usable()
        if why is None:
            return "zig"
        print(f"warning: the Zig-kernel port is unusable here ({why}); timing the torch path", file=sys.stderr)
    return "reference" if reference_package_root() is not None else "torch"


_CPU_IMPL_TEXT = {
    "reference": "the reference package's own torch CPU path (backend='torch'), unmodified",
    "torch": "numpy oracle of the reference torch CPU path",
    "zig": "C++ restatement of the reference's Zig CPU inference kernels, backend='zig'",
}


def _reference_module(w: Workload):
    """The workload's layer (or classifier) built from the reference package's own classes with
    their default torch backend, same seeds and dtype as the b200 arm."""
    root = reference_package_root()
    if str(root) not in sys.path:
        sys.path.append(str(root))
    import tropnn

    if w.classifier:
        cls = tropnn.TropLinear if w.kind == "trop_clf" else tropnn.PairwiseLinear
        dims = [w.in_features, w.hidden, w.out_features]
        model = _Classifier([cls(a, b, seed=i, **w.layer_kwargs) for i, (a, b) in enumerate(zip(dims[:-1], dims[1:]))])
        model.optimizer = torch.optim.Adam(model.parameters(), lr=1e-3)
        return model.train()
    cls = tropnn.PairwiseLinear if w.kind == "pairwise" else tropnn.TropLinear
    layer = cls(w.in_features, w.out_features, seed=0, **w.layer_kwargs)
    if w.dtype == "float16":
        layer = layer.half()
    return layer.train(w.train)


def time_reference_torch(w: Workload, sample_rows: int, *, reps: int | None = None, budget_s: float = 10.0,
                         warmup: int = 1) -> dict:
    """rows/s of the reference package's own torch path on ``sample_rows`` rows per step, in this
    process with torch's intra-op threads on every host core: eval = no_grad forward; train =
    zero grads, forward, backward of the upstream gradient; classifiers = forward, cross-entropy,
    backward, Adam step."""
    torch.set_num_threads(os.cpu_count() or 1)
    module = _reference_module(w)
    gen = torch.Generator().manual_seed(7)
    if w.classifier:
        x = torch.rand(sample_rows, w.in_features, generator=gen)
        g = torch.randint(0, w.out_features, (sample_rows,), generator=gen)
    else:
        x = torch.randn(sample_rows, w.in_features, generator=gen)
        g = torch.randn(sample_rows, 1, w.out_features, generator=gen)

    def step() -> None:
        if w.classifier:
            module.optimizer.zero_grad(set_to_none=True)
            torch.nn.functional.cross_entropy(module(x), g).backward()
            module.optimizer.step()
        elif w.train:
            for p in module.parameters():
                p.grad = None
            xi = x.detach().requires_grad_(True)
            module(xi).backward(g)
        else:
            with torch.no_grad():
                module(x)

    for _ in range(max(1, warmup)):
        step()
    done = 0
    t0 = time.perf_counter()
    while (reps is not None and done < reps) or (reps is None and (done == 0 or time.perf_counter() - t0 < budget_s)):
        step()
        done += 1
    dt = time.perf_counter() - t0
    return {"rows_per_s": sample_rows * done / dt, "seconds": dt, "steps": done, "threads": torch.get_num_threads()}


def _oracle_step(w: Workload, params: dict, layer, x: np.ndarray, g: np.ndarray, impl: str = "torch") -> None:
    import oracle

    if w.classifier:
        _oracle_classifier_step(w, params, x, g)
        return
    if impl == "zig":
        from oracle import native

        if w.kind == "pairwise":
            native.pairwise_eval(x, params, output_scale=layer.output_scale, threads=1)
        else:
            native.trop_linear_eval(x, params, code_scale=layer.code_scale, threads=1)
        return
    if w.kind == "pairwise":
        fwd = oracle.pairwise_forward(x, params["anchors"], params["thresholds"], params["lut"], output_scale=layer.output_scale)
        if w.train:
            oracle.pairwise_backward(
                g, fwd["indices"], fwd["margins"], params["anchors"], params["lut"], in_features=w.in_features,
                output_scale=layer.output_scale, use_min_margin_ste=layer.use_min_margin_ste, surrogate=layer.surrogate,
            )
        return
    fwd = oracle.trop_linear_forward(x, params, code_scale=layer.code_scale, training=w.train, param_dtype=w.dtype)
    if w.train:
        oracle.trop_linear_backward(g, x, params, fwd, code_scale=layer.code_scale, training=True, param_dtype=w.dtype)


_POOL_STATE: dict = {}


def _pool_init(workload: str, sample_rows: int, workers: int, impl: str = "torch") -> None:
    """Spawned CPU worker: one BLAS thread (one native thread), its own seeded parameters and
    row chunk."""
    from threadpoolctl import threadpool_limits

    torch.set_num_threads(1)
    _POOL_STATE["limits"] = threadpool_limits(limits=1)
    w = WORKLOADS[workload]
    if impl == "zig":
        from oracle import native

        native.load()
    gen = np.random.default_rng(7)
    if w.classifier:
        params, layer = _classifier_state(w), None
        x = gen.random((sample_rows, w.in_features), dtype=np.float32)
        g = gen.integers(0, w.out_features, sample_rows)
    else:
        params, layer = _oracle_params(w, impl)
        x = gen.standard_normal((sample_rows, w.in_features), dtype=np.float32)
        g = gen.standard_normal((sample_rows, w.out_features), dtype=np.float32)
    _POOL_STATE.update(w=w, params=params, layer=layer, x=x, g=g, impl=impl,
                       chunks=[c for c in np.array_split(np.arange(sample_rows), workers) if c.size])


def _pool_task(i: int) -> int:
    s = _POOL_STATE
    chunks = s["chunks"]
    if i < len(chunks):
        c = chunks[i]
        _oracle_step(s["w"], s["params"], s["layer"], s["x"][c], s["g"][c], s["impl"])
    return i


def time_cpu(w: Workload, sample_rows: int, workers: int, *, reps: int | None = None, budget_s: float = 10.0,
             warmup: int = 1, impl: str = "torch") -> dict:
    """rows/s of the oracle on ``sample_rows`` rows per step, the rows split over ``workers``
    spawn-started processes (one core each). Wall time of ``reps`` steps (or of as many
    steps as fit in ``budget_s``) after ``warmup`` steps."""
    import multiprocessing

    ctx = multiprocessing.get_context("spawn")
    if impl == "zig":
        from oracle import native

        native.build()  # before the workers start: they only load it
    with ctx.Pool(workers, initializer=_pool_init, initargs=(w.name, sample_rows, workers, impl)) as pool:
        for _ in range(max(1, warmup)):
            pool.map(_pool_task, range(workers), chunksize=1)
        done = 0
        t0 = time.perf_counter()
        while (reps is not None and done < reps) or (reps is None and (done == 0 or time.perf_counter() - t0 < budget_s)):
            pool.map(_pool_task, range(workers), chunksize=1)
            done += 1
        dt = time.perf_counter() - t0
    return {"rows_per_s": sample_rows * done / dt, "seconds": dt, "steps": done}


def cpu_baseline(w: Workload, budget_s: float, impl: str = "torch") -> dict:
    if impl == "reference":
        sample = w.ref_rows
        res = time_reference_torch(w, sample, budget_s=budget_s, warmup=1)
        return {
            "value": round(res["rows_per_s"], 1),
            "unit": "rows/s",
            "cores": res["threads"],
            "kind": "reference",
            "sample": f"{res['steps']} steps x {sample} rows of {w.name} ({_CPU_IMPL_TEXT[impl]}), "
            f"{res['seconds']:.1f} s, {res['threads']} torch threads",
        }
    workers = os.cpu_count() or 1
    sample = w.cpu_rows
    res = time_cpu(w, sample, workers, budget_s=budget_s, warmup=2, impl=impl)
    return {
        "value": round(res["rows_per_s"], 1),
        "unit": "rows/s",
        "cores": workers,
        "kind": "port",
        "sample": f"{res['steps']} steps x {sample} rows of {w.name} ({_CPU_IMPL_TEXT[impl]}), "
        f"{res['seconds']:.1f} s over {workers} single-threaded processes",
    }


def run_reference(args: argparse.Namespace, w: Workload) -> dict | None:
    rank, world, _ = _dist_env()
    if rank != 0:
        return None
    impl = cpu_impl_for(w, args.cpu_impl)
    if impl == "reference":
        sample = w.ref_rows
        res = time_reference_torch(w, sample, reps=args.steps, warmup=args.warmup)
        cores, kind = res["threads"], "reference"
        how = f"{res['threads']} torch threads in one process"
    else:
        cores = os.cpu_count() or 1
        sample = w.cpu_rows
        res = time_cpu(w, sample, cores, reps=args.steps, warmup=args.warmup, impl=impl)
        kind = "port"
        how = f"{cores} single-threaded processes"
    value = res["rows_per_s"]
    return {
        "metric": METRIC,
        "impl": "reference",
        "value": round(value, 1),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["seconds"] / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": w.scaling,
        "vs_baseline": None,
        "dtype": "f32" if w.dtype == "float32" else "f16 params / f32 accumulate",
        "data": "synthetic (seeded N(0,1) inputs and upstream grads; seeded default init)",
        "config": {"workload": w.description, "rows_per_step_sample": sample},
        "cpu_baseline": {
            "value": round(value, 1),
            "unit": "rows/s",
            "cores": cores,
            "kind": kind,
            "sample": f"{args.steps} steps x {sample} rows ({_CPU_IMPL_TEXT[impl]}, {how})",
        },
        "e2e": {"value": round(value, 1), "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="trop_cfg5_train")
    parser.add_argument(
        "--secondary", choices=["none", *sorted(WORKLOADS)], default="pairwise_cfg5_train",
        help="a second workload timed after the first (same GPUs, same K/W), reported under 'secondary' "
        "(default: the config 5 PairwiseLinear train step beside the config 5 TropLinear one)",
    )
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--cpu-budget-s", type=float, default=10.0, help="seconds of CPU-baseline timing (rank 0, N=1)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument(
        "--cpu-impl", choices=["auto", "reference", "torch", "zig"], default="auto",
        help="CPU path of the cpu_baseline leg and the reference arm: reference = the reference package's own "
        "torch path (installed under baseline/_ref); torch = numpy port of that path; zig = C++ restatement of "
        "its Zig inference kernels (eval workloads only); auto = the reference's faster CPU path on the workload",
    )
    parser.add_argument("--rows", type=int, default=0, help="override the row count (per GPU, or global for "
                        "strong-scaling workloads; profiling runs)")
    parser.add_argument(
        "--fuse-lut-allreduce", type=int, choices=[0, 1], default=0,
        help="with the peer all-reduce, average the Pairwise LUT gradient inside its kernel (1) or after the "
        "backward (0, the default: two GPUs, config 2, 101.3 us per step against 115.8 us fused)",
    )
    parser.add_argument(
        "--allreduce", choices=["auto", "peer", "nccl"], default="auto",
        help="gradient all-reduce at N>1: peer = the NVLink peer-memory kernel (up to 8 GPUs), nccl = NCCL, "
        "auto = peer up to 4 GPUs, NCCL above",
    )
    args = parser.parse_args(argv)
    if args.warmup < 3 and args.impl == "b200":
        parser.error("--warmup must be >= 3")
    import dataclasses

    def workload(name: str) -> Workload:
        w = WORKLOADS[name]
        if args.rows > 0:
            w = dataclasses.replace(w, rows_per_gpu=args.rows, description=f"{w.description} [rows overridden: {args.rows}]")
        return w

    w = workload(args.workload)
    _, world, local_rank = _dist_env()
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; reporting WORLD_SIZE", file=sys.stderr)

    if args.impl == "reference":
        line = run_reference(args, w)
    else:
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
        _init_dist(device, world)
        try:
            line = run_b200(args, w)
            if args.secondary != "none" and args.secondary != args.workload:
                second = run_b200(args, workload(args.secondary))
                if line is not None and second is not None:
                    line["secondary"] = {k: second[k] for k in (
                        "value", "unit", "ms_per_step", "scaling", "dtype", "config", "e2e", "e2e_modes",
                        "gpu_launches", "kernels", "roofline", "kernel_rooflines", "clocks")}
                    line["gpu_launches_secondary"] = second["gpu_launches"]
        finally:
            _end_dist(world)
        if line is not None and world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w, args.cpu_budget_s, cpu_impl_for(w, args.cpu_impl))
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
