"""FusedAdam: Faster-GS's optimizer interface (cluster/patches/fastergs_lean_adam.patch:251-307) with every
parameter group updated by ONE launch of adam_step_multi (csrc/adam.cu) instead of one launch per group, and the
lean options of that patch (visibility-sparse update, bfloat16 moments) through adam_step_multi_lean.

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
                ("exp_avg_sq", ctypes.c_void_p), ("n", ctypes.c_longlong), ("lr", ctypes.c_double)]


class _LeanGroup(ctypes.Structure):
    """Mirror of adam_lean_group in include/splat_b200.h."""

    _fields_ = [("param", ctypes.c_void_p), ("grad", ctypes.c_void_p), ("exp_avg", ctypes.c_void_p),
                ("exp_avg_sq", ctypes.c_void_p), ("n", ctypes.c_longlong), ("lr", ctypes.c_double),
                ("features", ctypes.c_int), ("lowp_moments", ctypes.c_int)]


MAX_GROUPS = 8


class FusedAdam(torch.optim.Adam):
    """Adam over single-tensor parameter groups, all groups in one kernel launch per step.

    The options of the reference's lean optimizer (cluster/patches/fastergs_lean_adam.patch:251-307), both off by
    default (then this is the original Faster-GS optimizer):
      sparse              only primitives visible in the last differentiable forward (n_touched_tiles > 0, handed
                          over by gs3d._Rasterize.last_visibility) are updated; the others keep their parameters
                          and moments for that step
      lowp_moment_groups  names of parameter groups whose exp_avg / exp_avg_sq are kept in bfloat16 (stochastic
                          rounding on write)
    and one of this build (off by default; with the dense update only):
      fuse_backward       when the six 3DGS tensors of a diff_rasterize call (means, scales, rotations, opacities,
                          sh0, sh_rest) are parameters of this optimizer, each alone in its group, the rasterizer's
                          backward leaves their preprocess backward to step(), which runs it fused with their Adam
                          update (gs3d_backward_preprocess_adam): their gradients are never written, so .grad stays
                          None for them after backward() unless other loss terms contributed (those gradients are
                          added inside the fused step). The parameters, moments and densification statistics are
                          bit-identical to the unfused path for one rendered view per step; with several views per
                          step all but the last are materialised into .grad when the next one arrives.
    """

    def __init__(self, params, lr, eps, betas=(0.9, 0.999), sparse: bool = False,
                 lowp_moment_groups: tuple = (), fuse_backward: bool = False) -> None:
        super().__init__(params=params, lr=lr, eps=eps, betas=betas)
        self.sparse = bool(sparse)
        self.lowp_moment_groups = set(lowp_moment_groups)
        self.lean = self.sparse or bool(self.lowp_moment_groups)
        self.n_dense_fallbacks = 0
        self.fuse_backward = bool(fuse_backward)
        self._pending = None  # (PendingBackward, the six parameter tensors)
        if self.fuse_backward and self.lean:
            raise RuntimeError("fuse_backward takes the dense update (no sparse / lowp_moment_groups)")
        from . import gs3d

        gs3d._Rasterize.track_visibility = self.sparse
        if self.fuse_backward:
            gs3d._Rasterize.fused_optimizer = self

    # ---- fused preprocess backward + Adam ----

    def _group_of(self, t: torch.Tensor):
        for group in self.param_groups:
            if len(group["params"]) == 1 and group["params"][0].data_ptr() == t.data_ptr() \
                    and group["params"][0].shape == t.shape:
                return group
        return None

    def _owns(self, six) -> bool:
        """True when the six rasterizer tensors are this optimizer's parameters (one per group, float32 CUDA,
        contiguous), so their preprocess backward can be deferred to step()."""
        if not self.fuse_backward:
            return False
        for t in six:
            if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()) or self._group_of(t) is None:
                return False
        return True

    def _defer(self, pending, six) -> None:
        if self._pending is not None:  # an earlier view of this step: its gradients go to .grad now
            earlier, tensors = self._pending
            grads = earlier.preprocess()
            for p, g in zip(self._params_of(tensors), grads):
                g = g.view(p.shape)
                p.grad = g if p.grad is None else p.grad + g
        self._pending = (pending, six)

    def _params_of(self, tensors):
        return [self._group_of(t)["params"][0] for t in tensors]

    def zero_grad(self, set_to_none: bool = True) -> None:  # noqa: D102
        self._pending = None
        super().zero_grad(set_to_none=set_to_none)

    @torch.no_grad()
    def _fused_step(self) -> set:
        pending, tensors = self._pending
        self._pending = None
        params = self._params_of(tensors)
        groups = [self._group_of(t) for t in tensors]
        exp_avg, exp_avg_sq, steps, lrs, grad_in = [], [], [], [], []
        for p, group in zip(params, groups):
            state = self.state[p]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0)
                state["exp_avg"] = torch.zeros_like(p)
                state["exp_avg_sq"] = torch.zeros_like(p)
            state["step"] += 1
            exp_avg.append(state["exp_avg"])
            exp_avg_sq.append(state["exp_avg_sq"])
            steps.append(int(state["step"].item()))
            lrs.append(float(group["lr"]))
            grad_in.append(p.grad)
        b1, b2 = groups[0]["betas"]
        eps = groups[0]["eps"]
        for group in groups[1:]:
            if tuple(group["betas"]) != (b1, b2) or group["eps"] != eps:
                raise RuntimeError("fuse_backward needs the same betas and eps in the six groups")
        pending.preprocess_adam(params, exp_avg, exp_avg_sq, lrs, steps, (b1, b2), eps, grad_in)
        return {id(p) for p in params}

    @torch.no_grad()
    def step(self, closure=None) -> None:  # noqa: D102
        if closure is not None:
            raise RuntimeError("FusedAdam does not take a closure")
        done = self._fused_step() if self._pending is not None else set()
        visibility = None
        if self.sparse:
            from . import gs3d

            visibility = gs3d._Rasterize.last_visibility
        by_key: dict[tuple, list] = {}
        masks: dict[tuple, torch.Tensor | None] = {}
        for group in self.param_groups:
            if len(group["params"]) != 1:
                raise RuntimeError("more than one tensor in group")
            param = group["params"][0]
            if id(param) in done or param.grad is None or param.numel() == 0:
                continue
            L.check_cuda("param", param, torch.float32)
            lowp = group.get("name") in self.lowp_moment_groups
            moment_dtype = torch.bfloat16 if lowp else param.dtype
            state = self.state[param]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0)
                state["exp_avg"] = torch.zeros_like(param, dtype=moment_dtype)
                state["exp_avg_sq"] = torch.zeros_like(param, dtype=moment_dtype)
            elif state["exp_avg"].dtype != moment_dtype:
                # densification concatenates float32 zeros to the moments, which promotes them; convert back
                state["exp_avg"] = state["exp_avg"].to(moment_dtype)
                state["exp_avg_sq"] = state["exp_avg_sq"].to(moment_dtype)
            state["step"] += 1
            grad = param.grad if param.grad.is_contiguous() else param.grad.contiguous()
            step = int(state["step"].item())
            if not self.lean:
                key = ("dense", step, *group["betas"], group["eps"], param.device)
                entry = _Group(param.data_ptr(), grad.data_ptr(), state["exp_avg"].data_ptr(),
                               state["exp_avg_sq"].data_ptr(), param.numel(), float(group["lr"]))
            else:
                vis = visibility
                if vis is not None and vis.numel() != param.shape[0]:
                    vis = None  # stale mask: this group falls back to the dense update
                    self.n_dense_fallbacks += 1
                key = ("lean", step, *group["betas"], group["eps"], param.device, None if vis is None else id(vis))
                masks[key] = vis
                entry = _LeanGroup(param.data_ptr(), grad.data_ptr(), state["exp_avg"].data_ptr(),
                                   state["exp_avg_sq"].data_ptr(), param.numel(), float(group["lr"]),
                                   param.numel() // max(param.shape[0], 1), int(lowp))
            entry._keep = grad
            by_key.setdefault(key, []).append(entry)
        for key, groups in by_key.items():
            kind, step, b1, b2, eps, dev = key[:6]
            stream = torch.cuda.current_stream(dev).cuda_stream
            for s in range(0, len(groups), MAX_GROUPS):
                chunk = groups[s:s + MAX_GROUPS]
                if kind == "dense":
                    arr = (_Group * len(chunk))(*chunk)
                    L.call("adam_step_multi", len(chunk), ctypes.addressof(arr), step, float(b1), float(b2),
                           float(eps), stream)
                else:
                    vis = masks[key]
                    arr = (_LeanGroup * len(chunk))(*chunk)
                    L.call("adam_step_multi_lean", len(chunk), ctypes.addressof(arr), step, float(b1), float(b2),
                           float(eps), L.ptr(vis), 0 if vis is None else vis.numel(), stream)


def adam_step(groups: list[tuple], step: int, betas=(0.9, 0.999), eps: float = 1e-15) -> None:
    """Functional form: groups = [(param, grad, exp_avg, exp_avg_sq, lr), ...] (CUDA float32, contiguous)."""
    if not groups:
        return
    arr = (_Group * len(groups))(*[_Group(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), float(lr))
                                   for p, g, m, v, lr in groups])
    L.call("adam_step_multi", len(groups), ctypes.addressof(arr), int(step), float(betas[0]), float(betas[1]),
           float(eps), L.stream_of(groups[0][0]))


def adam_step_lean(groups: list[tuple], step: int, visibility: torch.Tensor | None = None, betas=(0.9, 0.999),
                   eps: float = 1e-15) -> None:
    """Functional lean form (the reference's `_C.adam_step_sparse` for several groups at once): groups =
    [(param, grad, exp_avg, exp_avg_sq, lr), ...]; exp_avg / exp_avg_sq float32 or bfloat16 (stochastic rounding);
    visibility int32 [n_primitives] on the GPU or None."""
    if not groups:
        return
    entries = []
    for p, g, m, v, lr in groups:
        if m.dtype != v.dtype or m.dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError("moments must share a dtype, float32 or bfloat16")
        if visibility is not None and (visibility.dtype != torch.int32 or not visibility.is_cuda):
            raise RuntimeError("visibility must be int32 [n_primitives] on CUDA")
        entries.append(_LeanGroup(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), float(lr),
                                  p.numel() // max(p.shape[0], 1), int(m.dtype == torch.bfloat16)))
    arr = (_LeanGroup * len(entries))(*entries)
    L.call("adam_step_multi_lean", len(entries), ctypes.addressof(arr), int(step), float(betas[0]), float(betas[1]),
           float(eps), L.ptr(visibility), 0 if visibility is None else visibility.numel(), L.stream_of(groups[0][0]))
