"""Runs a golden case through the b200 layers on CUDA, returning fixture-keyed numpy results (test helper)."""

from __future__ import annotations

import numpy as np
import torch


def run_b200(layer: torch.nn.Module, arrays: dict[str, np.ndarray], meta: dict, device: str = "cuda") -> dict[str, np.ndarray]:
    layer = layer.to(device)
    layer.train(meta["train"])
    x = torch.from_numpy(arrays["x"]).to(device)
    out: dict[str, np.ndarray] = {}
    if meta["train"]:
        xg = x.clone().requires_grad_(True)
        y = layer(xg)
        g = torch.from_numpy(arrays["grad_out"]).to(device)
        (y * g).sum().backward()
        out["grad.x"] = xg.grad.cpu().numpy()
        for name, p in layer.named_parameters():
            out[f"has_grad.{name}"] = np.array(p.grad is not None)
            if p.grad is not None:
                out[f"grad.{name}"] = p.grad.float().cpu().numpy()
    else:
        with torch.no_grad():
            y = layer(x)
    torch.cuda.synchronize()
    out["y"] = y.detach().float().cpu().numpy()
    if layer._last_indices is not None:
        out["last_indices"] = layer._last_indices.cpu().numpy()
        out["last_margins"] = layer._last_margins.cpu().numpy()
    return out
