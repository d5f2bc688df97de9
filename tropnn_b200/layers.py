"""Drop-in ``TropLinear`` / ``PairwiseLinear`` for backend="b200".

Constructor arguments, parameter and buffer names, shapes, dtypes, ``state_dict`` keys
and the seeded initialisation order are those of the reference classes
(layers/tropical.py:21-79, layers/pairwise.py:18-68, layers/base.py:13-35), so a
``state_dict`` saved from the reference loads here unchanged and the same ``seed``
gives bit-identical parameters. The forward follows layers/base.py:64-84: 2-D input
becomes ``[B, 1, in]`` (the output stays 3-D), compute dtype is f32 for f16/bf16
input, and the route debug cache ``_last_indices``/``_last_margins`` is kept. The
routed part runs on the sm_100a kernels; any backend other than "b200" and any CPU
input raise, there is no fallback.

The forward bodies are module-agnostic functions (``trop_forward_b200``,
``pairwise_route_output_b200``) so that ``tropnn_b200.register`` can attach them to the
reference's own classes.
"""

from __future__ import annotations

import math
from typing import Literal

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from .ops import (
    EXACT_EVAL_MAX_IN,
    gemm_f32,
    gemm_f32_eligible,
    linear_f32_b200,
    linear_f32_eligible,
    linear_f32out_b200,
    linear_f32out_eligible,
    linear_f32out_shape_ok,
    pairwise_anchor_index,
    pairwise_b200,
    proj_eligible,
    trop_exact_eval_b200,
    trop_project_b200,
    trop_route_hidden_split,
    transpose_f32,
)

__all__ = [
    "PairwiseLinear",
    "RoutedLinearBase",
    "TropFanLinear",
    "TropLinear",
    "fan_forward_b200",
    "fan_generated_values",
    "pairwise_route_output_b200",
    "trop_forward_b200",
]

Backend = Literal["b200"]
_SURROGATES = ("fast_sigmoid_odd", "izhikevich")
MAX_COMPARISONS = 12


def _check_backend(backend: str) -> None:
    if backend != "b200":
        raise ValueError(
            f"tropnn_b200 layers only run backend='b200' (got {backend!r}); use the reference package for "
            "the torch/tilelang/triton/zig backends"
        )


def _compute_dtype(x: Tensor) -> torch.dtype:
    """layers/base.py:34-35."""
    return torch.float32 if x.dtype in {torch.float16, torch.bfloat16} else x.dtype


def _store_debug(layer: nn.Module, indices: Tensor, margins: Tensor) -> None:
    """layers/base.py:78-83: cache the last routes unless cache_route_debug is False.

    Packed (uint8/int16) route indices are kept as they are on this package's own layers,
    which widen them to the reference's int64 only when ``_last_indices`` is read; other
    modules (the reference classes under ``register``) get the int64 tensor at once.
    """
    if getattr(layer, "cache_route_debug", True):
        if indices.dtype != torch.int64 and isinstance(layer, RoutedLinearBase):
            layer._set_packed_indices(indices.detach())
        else:
            layer._last_indices = indices.detach().to(torch.int64)
        layer._last_margins = margins.detach()
    else:
        layer._last_indices = None
        layer._last_margins = None


def _require_cuda_input(x: Tensor, layer_name: str) -> None:
    if not x.is_cuda:
        raise ValueError(f"{layer_name} backend='b200' requires CUDA input tensors; there is no CPU fallback")


def _require_f32_compute(compute_dtype: torch.dtype, layer_name: str) -> None:
    if compute_dtype != torch.float32:
        raise TypeError(f"{layer_name} backend='b200' requires float32 compute dtype, got {compute_dtype}")


# ---------------------------------------------------------------------------
# module-agnostic forward bodies
# ---------------------------------------------------------------------------


def _exact_eval_params(layer: nn.Module, device: torch.device) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Effective weights of the exact eval path in f32 (layers/tropical_exact.py:257-291):
    router_eff = W P [H,K,in], router_bias, value_eff = c Wout^T [H,K,out], base = Wout P
    [out,in], cached per parameter version like the reference's _exact_eval_cache."""
    bias = layer.output_proj.bias
    key = (
        device,
        layer.proj.weight._version,
        layer.output_proj.weight._version,
        -1 if bias is None else bias._version,
        layer.router_weight._version,
        layer.router_bias._version,
        layer.code._version,
        layer.proj.weight.data_ptr(),
        layer.router_weight.data_ptr(),
        layer.code.data_ptr(),
    )
    cached = getattr(layer, "_b200_exact_eval_cache", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    f32 = torch.float32
    heads, cells, dim = layer.router_weight.shape
    with torch.no_grad():  # inference weights: the cache holds no autograd history
        proj = layer.proj.weight.to(device=device, dtype=f32).contiguous()
        w_out = layer.output_proj.weight.to(device=device, dtype=f32).contiguous()
        weight = layer.router_weight.to(device=device, dtype=f32).reshape(heads * cells, dim).contiguous()
        code = layer.code.to(device=device, dtype=f32).reshape(heads * cells, dim).contiguous()
        if gemm_f32_eligible(proj, w_out, weight, code):
            # f32 products on the tensor cores (3xTF32): W P and Wout P against P^T.
            proj_t = transpose_f32(proj)
            router_eff = gemm_f32(weight, proj_t, k=dim)
            value_eff = gemm_f32(code, w_out)
            base = gemm_f32(w_out, proj_t, k=dim)
        else:
            router_eff = torch.matmul(weight, proj)
            value_eff = torch.matmul(code, w_out.t())
            base = torch.matmul(w_out, proj)
        params = (
            router_eff.view(heads, cells, -1).contiguous(),
            layer.router_bias.to(device=device, dtype=f32).contiguous(),
            value_eff.view(heads, cells, -1).contiguous(),
            base.contiguous(),
        )
    layer._b200_exact_eval_cache = (key, params)
    return params


def _trop_exact_eval_b200(layer: nn.Module, x: Tensor) -> Tensor:
    """TropLinear forward with ``exact_fused="eval"`` in eval under no_grad
    (layers/tropical_exact.py:297-358): x in the compute dtype (not rounded to the parameters),
    scores against W P on the route kernel, y = x (Wout P)^T + b_out (the reference's f32 matmul,
    here the 3xTF32 tensor-core product) plus code_scale * sum_h (c Wout^T)[h, winner] on the
    code-sum kernel."""
    input_dtype = x.dtype
    compute_dtype = _compute_dtype(x)
    _require_f32_compute(compute_dtype, "TropLinear")
    batch, steps, in_features = x.shape
    x_flat = x.to(compute_dtype).reshape(batch * steps, in_features).contiguous()
    router_eff, router_bias, value_eff, base = _exact_eval_params(layer, x.device)
    bias = layer.output_proj.bias
    if gemm_f32_eligible(x_flat, base):
        # x (Wout P)^T + b_out on the f32 tensor-core product (3xTF32).
        base_out = gemm_f32(x_flat, base, None if bias is None else bias.to(device=x.device, dtype=compute_dtype))
    else:
        base_out = torch.matmul(x_flat, base.t())
        if bias is not None:
            base_out = base_out + bias.to(device=x.device, dtype=compute_dtype)
    y, winner, margins = trop_exact_eval_b200(
        x_flat, router_eff, router_bias, value_eff, base_out, code_scale=layer.code_scale,
        keep_margins=getattr(layer, "cache_route_debug", True),
    )
    _store_debug(layer, winner.view(batch, steps, -1), margins.view(batch, steps, -1) if margins.numel() else margins)
    return y.view(batch, steps, -1).to(dtype=input_dtype)


def trop_forward_b200(layer: nn.Module, x: Tensor) -> Tensor:
    """Full TropLinear forward on sm_100a for any module with the TropLinear attributes.

    The projection (tropical.py:96-99) runs on the b200 tensor-core projection kernel for
    half-precision weights (ops.trop_project_b200) and on the 3xTF32 tensor-core product for
    f32 weights (ops.linear_f32_b200); the route scores, top-2, code sum and their backward are
    the b200 kernels (ops.trop_route_hidden_split); the output map (tropical.py:140-146) is the
    b200 tensor-core linear map for half-precision weights (ops.linear_f32out_b200) or the
    3xTF32 product for f32 weights. Widths the kernels do not tile (inputs not a multiple of 4
    floats wide) use torch.
    """
    if x.ndim == 2:
        x = x.unsqueeze(1)
    _require_cuda_input(x, "TropLinear")
    if (
        getattr(layer, "exact_fused", "off") == "eval"
        and not layer.training
        and not torch.is_grad_enabled()
        and layer.in_features <= EXACT_EVAL_MAX_IN
    ):
        # layers/tropical.py:92: the reassociated eval path (wider inputs keep the default
        # path, the same function up to rounding).
        return _trop_exact_eval_b200(layer, x)
    return _routed_code_forward_b200(layer, x, layer.router_weight, layer.router_bias, layer.code, "TropLinear")


def _routed_code_forward_b200(
    layer: nn.Module, x: Tensor, router_weight: Tensor, router_bias: Tensor, code: Tensor, layer_name: str
) -> Tensor:
    """Projection, tropical routing with the selected-code sum, output map: the part TropLinear
    (layers/tropical.py:89-99, :131-146) and TropFanLinear (layers/fan.py:96-99, :201-222, :276-330)
    share; TropFanLinear's router is its sites and lifting and its code its generated values."""
    input_dtype = x.dtype
    compute_dtype = _compute_dtype(x)
    _require_f32_compute(compute_dtype, layer_name)
    if proj_eligible(x, layer.proj.weight):
        # Half-precision projection weight: the tensor-core projection kernel rounds x on chip.
        z = trop_project_b200(x, layer.proj.weight)
    elif linear_f32_eligible(x.to(torch.float32), layer.proj.weight):
        # f32 projection weight: the reference's f32 GEMM as 3xTF32 on the tensor cores.
        z = linear_f32_b200(x.to(torch.float32), layer.proj.weight, None)
    else:
        z = layer.proj(x.to(dtype=layer.proj.weight.dtype))
    # The reference upcasts z to the compute dtype (tropical.py:99); with half-precision
    # parameters the b200 op takes z in that dtype instead (the upcast is exact and happens
    # in-kernel), which lets the route scores run on the tensor cores.
    latent = z if z.dtype in (torch.float16, torch.bfloat16) and z.dtype == router_weight.dtype else z.to(compute_dtype)
    out_weight = layer.output_proj.weight
    # Half-precision output weight of the code dtype: the code sum's epilogue also writes the
    # [hi | lo] split of hidden that the output map's tensor-core product reads.
    fuse_split = (
        out_weight.dtype == code.dtype
        and out_weight.dtype in (torch.float16, torch.bfloat16)
        and out_weight.is_cuda
        and linear_f32out_shape_ok(out_weight.shape[0], out_weight.shape[1])
        and out_weight.shape[1] == code.shape[-1]
    )
    hidden, winner, margins, hidden_split = trop_route_hidden_split(
        latent,
        router_weight,
        router_bias,
        code,
        code_scale=layer.code_scale,
        training=layer.training,
        keep_margins=getattr(layer, "cache_route_debug", True),
        split_dtype=out_weight.dtype if fuse_split else None,
    )
    bias = layer.output_proj.bias
    if linear_f32out_eligible(hidden, out_weight):
        # Half-precision output weight: the f32 product on the tensor cores (split f32
        # hidden, bias fused), the reference's f32 math in the backward.
        output = linear_f32out_b200(hidden, out_weight, bias, hidden_split=hidden_split)
    elif linear_f32_eligible(hidden, layer.output_proj.weight) and (bias is None or bias.dtype == torch.float32):
        # f32 output weight: the reference's f32 F.linear as 3xTF32 on the tensor cores.
        output = linear_f32_b200(hidden, layer.output_proj.weight, bias)
    else:
        weight = layer.output_proj.weight.to(dtype=compute_dtype)
        output = torch.matmul(hidden, weight.t())
        if bias is not None:
            output = output + bias.to(dtype=compute_dtype)
    _store_debug(layer, winner, margins)
    return output.to(dtype=input_dtype)


def fan_generated_values(layer: nn.Module, compute_dtype: torch.dtype) -> Tensor:
    """TropFanLinear's value table [heads, cells, code_dim] (layers/fan.py:159-171), in the
    compute dtype from the parameters: "site" mode scales each unit-normalised site by its
    value_scale, "basis" mode is value_coeff times value_basis. A parameter-sized step
    (independent of the batch), kept differentiable so that autograd carries the code-sum
    kernel's value gradient back into sites / value_scale / value_coeff / value_basis."""
    if layer.fan_value_mode == "site":
        unit = F.normalize(layer.sites.to(compute_dtype), dim=-1, eps=1e-12)
        return unit * layer.value_scale.to(compute_dtype).unsqueeze(-1)
    return torch.einsum("hkr,rd->hkd", layer.value_coeff.to(compute_dtype), layer.value_basis.to(compute_dtype))


def fan_forward_b200(layer: nn.Module, x: Tensor) -> Tensor:
    """TropFanLinear forward on sm_100a for any module with the TropFanLinear attributes
    (layers/fan.py:276-330): the TropLinear path with the sites and lifting as the router and
    the generated values as the code table (scores, top-2, min-face mix and selected-value sum
    on the b200 kernels, as are the projection and the output map)."""
    if x.ndim == 2:
        x = x.unsqueeze(1)
    _require_cuda_input(x, "TropFanLinear")
    if layer.fan_recovery_mode != "untied":
        raise RuntimeError(
            "TropFanLinear fan_recovery_mode='tied' is only supported by the scaling benchmark tied recovery wrapper"
        )
    compute_dtype = _compute_dtype(x)
    values = fan_generated_values(layer, compute_dtype)
    # The route kernels take the code table in the router's dtype: half-precision layers round
    # the f32 values to it (2^-11 relative for f16, inside the half-precision tolerance).
    return _routed_code_forward_b200(
        layer, x, layer.sites, layer.lifting, values.to(layer.sites.dtype), "TropFanLinear"
    )


def _anchor_index(layer: nn.Module, anchors: Tensor) -> tuple[Tensor, Tensor]:
    """Inverse anchor map cached per (device, anchors version), like the reference's
    version-keyed parameter caches (layers/pairwise.py:82-92)."""
    key = (anchors.device, anchors.data_ptr(), anchors._version, tuple(anchors.shape))
    cached = getattr(layer, "_b200_anchor_index", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    lo = int(anchors.min())
    hi = int(anchors.max())
    if lo < 0 or hi >= layer.in_features:
        raise IndexError(f"PairwiseLinear anchors must lie in [0, {layer.in_features}), found [{lo}, {hi}]")
    index = pairwise_anchor_index(anchors, layer.in_features)
    layer._b200_anchor_index = (key, index)
    return index


def pairwise_route_output_b200(layer: nn.Module, latent: Tensor, training: bool) -> tuple[Tensor, Tensor, Tensor]:
    """PairwiseLinear ``_route_output`` on sm_100a, with ``output_scale`` already applied.

    The straight-through correction is live only when training and latent or thresholds
    need a gradient (layers/pairwise.py:245).
    """
    _require_cuda_input(latent, "PairwiseLinear")
    _require_f32_compute(latent.dtype, "PairwiseLinear")
    anchors = layer.anchors
    if anchors.device != latent.device:
        anchors = anchors.to(device=latent.device)
    ste = bool(training and (latent.requires_grad or layer.thresholds.requires_grad))
    return pairwise_b200(
        latent,
        anchors,
        layer.thresholds,
        layer.lut,
        use_min_margin_ste=layer.use_min_margin_ste,
        surrogate=layer.surrogate,
        output_scale=layer.output_scale,
        ste=ste,
        anchor_index=_anchor_index(layer, anchors),
    )


def pairwise_forward_b200(layer: nn.Module, x: Tensor) -> Tensor:
    """layers/base.py:64-84 for PairwiseLinear, with output_scale fused into the kernels."""
    if x.ndim == 2:
        x = x.unsqueeze(1)
    _require_cuda_input(x, "PairwiseLinear")
    input_dtype = x.dtype
    compute_dtype = _compute_dtype(x)
    _require_f32_compute(compute_dtype, "PairwiseLinear")
    latent = x.to(compute_dtype)
    output, indices, margins = pairwise_route_output_b200(layer, latent, layer.training)
    _store_debug(layer, indices, margins)
    return output.to(dtype=input_dtype)


# ---------------------------------------------------------------------------
# modules
# ---------------------------------------------------------------------------


class RoutedLinearBase(nn.Module):
    """Shell of the routed layers (layers/base.py:13-35): sizes, backend, output scale
    and the route debug cache."""

    def __init__(self, in_features: int, out_features: int, *, backend: Backend = "b200", output_scale: float = 1.0) -> None:
        super().__init__()
        if in_features < 1:
            raise ValueError(f"in_features must be >= 1, got {in_features}")
        if out_features < 1:
            raise ValueError(f"out_features must be >= 1, got {out_features}")
        _check_backend(backend)
        self.in_features = in_features
        self.out_features = out_features
        self.backend = backend
        self.output_scale = output_scale
        self._last_indices: Tensor | None = None
        self._last_margins: Tensor | None = None

    def _compute_dtype(self, x: Tensor) -> torch.dtype:
        return _compute_dtype(x)

    # Route debug cache. `_last_indices` reads as the reference's int64 tensor; when the
    # kernels hand over packed routes the widening copy is made on first read only.
    @property
    def _last_indices(self) -> Tensor | None:
        packed = self.__dict__.get("_b200_packed_indices")
        if packed is not None:
            self.__dict__["_b200_indices"] = packed.to(torch.int64)
            self.__dict__["_b200_packed_indices"] = None
        return self.__dict__.get("_b200_indices")

    @_last_indices.setter
    def _last_indices(self, value: Tensor | None) -> None:
        self.__dict__["_b200_indices"] = value
        self.__dict__["_b200_packed_indices"] = None

    def _set_packed_indices(self, packed: Tensor) -> None:
        self.__dict__["_b200_indices"] = None
        self.__dict__["_b200_packed_indices"] = packed


class TropLinear(RoutedLinearBase):
    """Tropical code layer with hard head routing and a shared output map, on sm_100a."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        *,
        heads: int = 32,
        cells: int = 4,
        code_dim: int = 32,
        backend: Backend = "b200",
        seed: int = 0,
        code_init_std: float = 0.02,
        use_output_scaling: bool = True,
        cpu_param_dtype: Literal["f32", "f16"] = "f32",
        exact_fused: Literal["off", "eval", "train"] = "off",
        score_route_max_bytes: int | None = None,
        cache_route_debug: bool = True,
    ) -> None:
        if heads < 1:
            raise ValueError(f"heads must be >= 1, got {heads}")
        if cells < 2:
            raise ValueError(f"cells must be >= 2, got {cells}")
        if code_dim < 1:
            raise ValueError(f"code_dim must be >= 1, got {code_dim}")
        if cpu_param_dtype not in {"f32", "f16"}:
            raise ValueError(f"cpu_param_dtype must be 'f32' or 'f16', got {cpu_param_dtype!r}")
        if exact_fused not in {"off", "eval", "train"}:
            raise ValueError(f"exact_fused must be 'off', 'eval', or 'train', got {exact_fused!r}")
        if score_route_max_bytes is not None and score_route_max_bytes < 0:
            raise ValueError(f"score_route_max_bytes must be >= 0 when set, got {score_route_max_bytes}")
        super().__init__(in_features, out_features, backend=backend, output_scale=1.0)
        self.heads = heads
        self.cells = cells
        self.code_dim = code_dim
        self.code_scale = 1.0 / math.sqrt(heads) if use_output_scaling else 1.0
        self.cpu_param_dtype = cpu_param_dtype
        # "eval" selects the reassociated eval path (effective weights, trop_forward_b200);
        # "train" and "off" run the fused b200 route, whose training backward already is the
        # exact min-face one (scores never materialised).
        self.exact_fused = exact_fused
        self.score_route_max_bytes = score_route_max_bytes
        self.cache_route_debug = cache_route_debug

        # Seeded initialisation in the reference's RNG order (layers/tropical.py:66-79).
        torch.manual_seed(seed)
        self.proj = nn.Linear(in_features, code_dim, bias=False)
        nn.init.normal_(self.proj.weight, mean=0.0, std=1.0 / math.sqrt(max(1, in_features)))
        router_std = 1.0 / math.sqrt(max(1, code_dim))
        self.router_weight = nn.Parameter(torch.randn(heads, cells, code_dim) * router_std)
        self.router_bias = nn.Parameter(torch.zeros(heads, cells))
        self.code = nn.Parameter(torch.randn(heads, cells, code_dim) * code_init_std)
        self.output_proj = nn.Linear(code_dim, out_features)
        nn.init.kaiming_uniform_(self.output_proj.weight, a=math.sqrt(5))
        if self.output_proj.bias is not None:
            fan_in = self.output_proj.weight.shape[1]
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.output_proj.bias, -bound, bound)

    def extra_repr(self) -> str:
        return (
            f"in_features={self.in_features}, out_features={self.out_features}, heads={self.heads}, "
            f"cells={self.cells}, code_dim={self.code_dim}, backend={self.backend!r}, cpu_param_dtype={self.cpu_param_dtype!r}, "
            f"exact_fused={self.exact_fused!r}, score_route_max_bytes={self.score_route_max_bytes!r}, "
            f"cache_route_debug={self.cache_route_debug!r}"
        )

    def forward(self, x: Tensor) -> Tensor:
        return trop_forward_b200(self, x)


FAN_VALUE_MODES = ("site", "basis")
FAN_RECOVERY_MODES = ("untied", "tied")


class TropFanLinear(RoutedLinearBase):
    """Tropical normal-fan layer (layers/fan.py:21-330) on sm_100a: routing sites with a
    lifting define the tropical polynomial, and the values the winning cells contribute are
    generated from the sites (``fan_value_mode="site"``: unit site times value_scale) or from
    a shared rank-``fan_basis_rank`` basis (``"basis"``: value_coeff times value_basis) instead
    of a free code table."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        *,
        heads: int = 32,
        cells: int = 4,
        code_dim: int = 32,
        backend: Backend = "b200",
        seed: int = 0,
        value_init_std: float = 0.02,
        fan_value_mode: Literal["site", "basis"] = "site",
        fan_basis_rank: int = 16,
        fan_recovery_mode: Literal["untied", "tied"] = "untied",
        use_output_scaling: bool = True,
        cpu_param_dtype: Literal["f32", "f16"] = "f32",
    ) -> None:
        if heads < 1:
            raise ValueError(f"heads must be >= 1, got {heads}")
        if cells < 2:
            raise ValueError(f"cells must be >= 2, got {cells}")
        if code_dim < 1:
            raise ValueError(f"code_dim must be >= 1, got {code_dim}")
        if fan_value_mode not in FAN_VALUE_MODES:
            raise ValueError(f"fan_value_mode must be one of {FAN_VALUE_MODES}, got {fan_value_mode!r}")
        if fan_recovery_mode not in FAN_RECOVERY_MODES:
            raise ValueError(f"fan_recovery_mode must be one of {FAN_RECOVERY_MODES}, got {fan_recovery_mode!r}")
        if fan_basis_rank < 1:
            raise ValueError(f"fan_basis_rank must be >= 1, got {fan_basis_rank}")
        if cpu_param_dtype not in {"f32", "f16"}:
            raise ValueError(f"cpu_param_dtype must be 'f32' or 'f16', got {cpu_param_dtype!r}")
        super().__init__(in_features, out_features, backend=backend, output_scale=1.0)
        self.heads = heads
        self.cells = cells
        self.code_dim = code_dim
        self.code_scale = 1.0 / math.sqrt(heads) if use_output_scaling else 1.0
        self.fan_value_mode = fan_value_mode
        self.fan_basis_rank = fan_basis_rank
        self.fan_recovery_mode = fan_recovery_mode
        self.cpu_param_dtype = cpu_param_dtype

        # Seeded initialisation in the reference's RNG order (layers/fan.py:87-103).
        torch.manual_seed(seed)
        self.proj = nn.Linear(in_features, code_dim, bias=False)
        nn.init.normal_(self.proj.weight, mean=0.0, std=1.0 / math.sqrt(max(1, in_features)))
        site_std = 1.0 / math.sqrt(max(1, code_dim))
        self.sites = nn.Parameter(torch.randn(heads, cells, code_dim) * site_std)
        self.lifting = nn.Parameter(torch.zeros(heads, cells))
        if fan_value_mode == "site":
            self.value_scale = nn.Parameter(torch.randn(heads, cells) * value_init_std)
            self.value_coeff = None
            self.value_basis = None
        else:
            self.value_scale = None
            self.value_coeff = nn.Parameter(
                torch.randn(heads, cells, fan_basis_rank) * value_init_std / math.sqrt(fan_basis_rank)
            )
            self.value_basis = nn.Parameter(torch.randn(fan_basis_rank, code_dim) / math.sqrt(max(1, code_dim)))
        self.output_proj = nn.Linear(code_dim, out_features)
        nn.init.kaiming_uniform_(self.output_proj.weight, a=math.sqrt(5))
        if self.output_proj.bias is not None:
            fan_in = self.output_proj.weight.shape[1]
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.output_proj.bias, -bound, bound)

    def extra_repr(self) -> str:
        return (
            f"in_features={self.in_features}, out_features={self.out_features}, heads={self.heads}, "
            f"cells={self.cells}, code_dim={self.code_dim}, fan_value_mode={self.fan_value_mode!r}, "
            f"fan_basis_rank={self.fan_basis_rank}, fan_recovery_mode={self.fan_recovery_mode!r}, backend={self.backend!r}, "
            f"cpu_param_dtype={self.cpu_param_dtype!r}"
        )

    def generated_values(self, *, input_device: torch.device | None = None, compute_dtype: torch.dtype | None = None) -> Tensor:
        """The value table [heads, cells, code_dim] (layers/fan.py:159-171)."""
        values = fan_generated_values(self, self.sites.dtype if compute_dtype is None else compute_dtype)
        return values if input_device is None else values.to(input_device)

    def forward(self, x: Tensor) -> Tensor:
        return fan_forward_b200(self, x)


class PairwiseLinear(RoutedLinearBase):
    """Pairwise-comparator LUT layer with min-margin (or full) STE, on sm_100a."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        *,
        tables: int = 16,
        comparisons: int = 4,
        backend: Backend = "b200",
        seed: int = 0,
        lut_init_std: float = 0.02,
        use_min_margin_ste: bool = True,
        use_output_scaling: bool = True,
        surrogate: str = "fast_sigmoid_odd",
        cpu_lut_dtype: Literal["f32", "f16"] = "f32",
    ) -> None:
        if tables < 1:
            raise ValueError(f"tables must be >= 1, got {tables}")
        if comparisons < 1:
            raise ValueError(f"comparisons must be >= 1, got {comparisons}")
        if comparisons > MAX_COMPARISONS:
            raise ValueError(f"backend='b200' supports comparisons <= {MAX_COMPARISONS}, got {comparisons}")
        _check_backend(backend)
        if cpu_lut_dtype not in {"f32", "f16"}:
            raise ValueError(f"cpu_lut_dtype must be 'f32' or 'f16', got {cpu_lut_dtype!r}")
        if surrogate not in _SURROGATES:
            raise ValueError(f"unsupported surrogate {surrogate!r}")
        output_scale = 1.0 / math.sqrt(tables) if use_output_scaling else 1.0
        super().__init__(in_features, out_features, backend=backend, output_scale=output_scale)
        self.tables = tables
        self.comparisons = comparisons
        self.table_size = 1 << comparisons
        self.use_min_margin_ste = use_min_margin_ste
        self.surrogate = surrogate
        self.cpu_lut_dtype = cpu_lut_dtype

        # Seeded initialisation in the reference's RNG order (layers/pairwise.py:55-68):
        # one scalar randint per anchor side, redrawing b while it equals a.
        torch.manual_seed(seed)
        anchors = torch.zeros(tables, comparisons, 2, dtype=torch.long)
        for table_idx in range(tables):
            for comp_idx in range(comparisons):
                first = torch.randint(0, in_features, (1,)).item()
                second = torch.randint(0, in_features, (1,)).item()
                while second == first:
                    second = torch.randint(0, in_features, (1,)).item()
                anchors[table_idx, comp_idx, 0] = first
                anchors[table_idx, comp_idx, 1] = second
        self.register_buffer("anchors", anchors)
        self.thresholds = nn.Parameter(torch.zeros(tables, comparisons))
        self.lut = nn.Parameter(torch.randn(tables, self.table_size, out_features) * lut_init_std)
        self.register_buffer("powers", 2 ** torch.arange(comparisons, dtype=torch.long))

    def extra_repr(self) -> str:
        return (
            f"in_features={self.in_features}, out_features={self.out_features}, tables={self.tables}, "
            f"comparisons={self.comparisons}, backend={self.backend!r}, use_min_margin_ste={self.use_min_margin_ste}, "
            f"surrogate={self.surrogate!r}, cpu_lut_dtype={self.cpu_lut_dtype!r}"
        )

    def forward(self, x: Tensor) -> Tensor:
        return pairwise_forward_b200(self, x)
