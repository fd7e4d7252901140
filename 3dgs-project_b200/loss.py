"""Fused L1 + SSIM training loss on the GPU (csrc/ssim.cu), with the call shapes of the fused-ssim package the
reference's trainer uses (`fused_ssim(img1, img2, padding="same", train=True)`, the mean SSIM, differentiable in
img1) and of 3DGS's combined loss ((1 - lambda) L1 + lambda (1 - SSIM), lambda = 0.2 by default).
"""
from __future__ import annotations

import torch

from . import _lib as L


def _shape(img: torch.Tensor, gt: torch.Tensor) -> tuple[int, int, int, int]:
    L.check_cuda("img", img, torch.float32)
    L.check_cuda("gt", gt, torch.float32)
    if img.shape != gt.shape or img.dim() not in (3, 4):
        raise RuntimeError(f"images must share a [C,H,W] or [B,C,H,W] shape, got {tuple(img.shape)} and "
                           f"{tuple(gt.shape)}")
    return tuple(img.shape) if img.dim() == 4 else (1, *img.shape)


def _padding(padding: str) -> int:
    if padding not in ("same", "valid"):
        raise ValueError("padding must be 'same' or 'valid'")
    return int(padding == "valid")


class _L1SSIM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img, gt, lam: float, valid: int, want_ssim: bool):
        img, gt = img.contiguous(), gt.contiguous()
        B, C, H, W = _shape(img, gt)
        ws = torch.empty(L.query("splat_l1_ssim_workspace_size", B, C, H, W), dtype=torch.uint8, device=img.device)
        out = torch.empty(2, dtype=torch.float32, device=img.device)  # loss, mean SSIM
        L.call("splat_l1_ssim_forward", L.ptr(img), L.ptr(gt), B, C, H, W, float(lam), valid, L.ptr(out[0:1]),
               L.ptr(out[1:2]), L.ptr(ws), ws.numel(), L.stream_of(img))
        ctx.save_for_backward(img, gt, ws)
        ctx.args = (B, C, H, W, float(lam), valid, want_ssim)
        return out[1] if want_ssim else out[0]

    @staticmethod
    def backward(ctx, grad_out):
        img, gt, ws = ctx.saved_tensors
        B, C, H, W, lam, valid, want_ssim = ctx.args
        # mean SSIM = 1 - loss when lambda = 1, so its gradient is the loss gradient negated
        g = (-grad_out if want_ssim else grad_out).detach().to(torch.float32).reshape(1).contiguous()
        grad = torch.empty_like(img)
        L.call("splat_l1_ssim_backward", L.ptr(img), L.ptr(gt), B, C, H, W, lam, valid, L.ptr(g), L.ptr(grad),
               L.ptr(ws), ws.numel(), L.stream_of(img))
        return grad, None, None, None, None


def l1_ssim_loss(img: torch.Tensor, gt: torch.Tensor, lambda_dssim: float = 0.2, padding: str = "same"):
    """(1 - lambda_dssim) mean|img - gt| + lambda_dssim (1 - mean SSIM(img, gt)); differentiable in img."""
    return _L1SSIM.apply(img, gt, float(lambda_dssim), _padding(padding), False)


def fused_ssim(img1: torch.Tensor, img2: torch.Tensor, padding: str = "same", train: bool = True):
    """Mean SSIM of img1 against img2 (fused-ssim's call), differentiable in img1. `train` is accepted for the
    same signature; the derivative maps are always kept (they cost one pass)."""
    return _L1SSIM.apply(img1, img2, 1.0, _padding(padding), True)
