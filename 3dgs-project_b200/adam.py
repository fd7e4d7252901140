"""FusedAdam: Faster-GS's optimizer interface (cluster/patches/fastergs_lean_adam.patch:251-307) with every
parameter group updated by ONE launch of adam_step_multi (csrc/adam.cu) instead of one launch per group.

State is the torch.optim.Adam layout ('step', 'exp_avg', 'exp_avg_sq' per parameter), so state_dict()
round-trips with torch's Adam and with checkpoints written by the reference's trainer.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L


class _Group(ctypes.Structure):
    """Mirror of adam_group in include/splat_b200.h."""

    _fields_ = [("param", ctypes.c_void_p), ("grad", ctypes.c_void_p), ("exp_avg", ctypes.c_void_p),
                ("exp_avg_sq", ctypes.c_void_p), ("n", ctypes.c_longlong), ("lr", ctypes.c_float)]


MAX_GROUPS = 8


class FusedAdam(torch.optim.Adam):
    """Adam over single-tensor parameter groups, all groups in one kernel launch per step."""

    def __init__(self, params, lr, eps, betas=(0.9, 0.999)) -> None:
        super().__init__(params=params, lr=lr, eps=eps, betas=betas)

    @torch.no_grad()
    def step(self, closure=None) -> None:  # noqa: D102
        if closure is not None:
            raise RuntimeError("FusedAdam does not take a closure")
        by_key: dict[tuple, list] = {}
        for group in self.param_groups:
            if len(group["params"]) != 1:
                raise RuntimeError("more than one tensor in group")
            param = group["params"][0]
            if param.grad is None or param.numel() == 0:
                continue
            L.check_cuda("param", param, torch.float32)
            state = self.state[param]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0)
                state["exp_avg"] = torch.zeros_like(param)
                state["exp_avg_sq"] = torch.zeros_like(param)
            state["step"] += 1
            grad = param.grad if param.grad.is_contiguous() else param.grad.contiguous()
            key = (int(state["step"].item()), *group["betas"], group["eps"], param.device)
            by_key.setdefault(key, []).append(_Group(param.data_ptr(), grad.data_ptr(), state["exp_avg"].data_ptr(),
                                                     state["exp_avg_sq"].data_ptr(), param.numel(),
                                                     float(group["lr"])))
            by_key[key][-1]._keep = grad
        for (step, b1, b2, eps, dev), groups in by_key.items():
            for s in range(0, len(groups), MAX_GROUPS):
                chunk = groups[s:s + MAX_GROUPS]
                arr = (_Group * len(chunk))(*chunk)
                L.call("adam_step_multi", len(chunk), ctypes.addressof(arr), step, float(b1), float(b2), float(eps),
                       torch.cuda.current_stream(dev).cuda_stream)


def adam_step(groups: list[tuple], step: int, betas=(0.9, 0.999), eps: float = 1e-15) -> None:
    """Functional form: groups = [(param, grad, exp_avg, exp_avg_sq, lr), ...] (CUDA float32, contiguous)."""
    if not groups:
        return
    arr = (_Group * len(groups))(*[_Group(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), float(lr))
                                   for p, g, m, v, lr in groups])
    L.call("adam_step_multi", len(groups), ctypes.addressof(arr), int(step), float(betas[0]), float(betas[1]),
           float(eps), L.stream_of(groups[0][0]))
