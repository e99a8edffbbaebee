"""Training-step losses on the GPU.

:func:`l1_loss` is the photometric L1 term of the reference's training step
(``training/train.py:140``: ``(image - target).abs().mean()``) as two fused
kernels: the forward reads image and target once, the backward writes the
whole gradient image -- zeros in the tile padding included -- in one pass,
where torch runs about ten elementwise kernels (subtract, abs, mean, and
their backward: sign, scale, the zero-filled slice gradient and its copy).
The gradient values are torch's bit for bit; the loss value is a
deterministic reduction that can differ from torch's mean in the last bits.
"""

from __future__ import annotations

import ctypes

import torch

from . import native


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _check(image: torch.Tensor, target: torch.Tensor) -> None:
    if not (image.is_cuda and target.is_cuda):
        raise RuntimeError("l1_loss runs on CUDA devices only (there is no CPU path)")
    if image.device != target.device:
        raise RuntimeError(f"image on {image.device}, target on {target.device}")
    if image.dim() != 3 or target.dim() != 3 or image.shape[2] != target.shape[2]:
        raise ValueError(f"expected [H, W, C] image and target, got {tuple(image.shape)} and "
                         f"{tuple(target.shape)}")
    if target.shape[0] > image.shape[0] or target.shape[1] > image.shape[1]:
        raise ValueError(f"target {tuple(target.shape)} is larger than the image "
                         f"{tuple(image.shape)}")


class _L1Loss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, image: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        image = image.detach().to(torch.float32).contiguous()
        target = target.detach().to(torch.float32).contiguous()
        lib = native.lib()
        height, width, channels = image.shape
        scratch = torch.empty((int(lib.gs_l1_loss_scratch_floats()),), dtype=torch.float32,
                              device=image.device)
        loss = torch.empty((), dtype=torch.float32, device=image.device)
        with torch.cuda.device(image.device):
            stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            native.check(lib.gs_l1_loss(_ptr(image), height, width, channels, _ptr(target),
                                        target.shape[0], target.shape[1], _ptr(scratch),
                                        _ptr(loss), stream), "gs_l1_loss")
        ctx.save_for_backward(image, target)
        return loss

    @staticmethod
    def backward(ctx, grad_loss: torch.Tensor):
        image, target = ctx.saved_tensors
        grad_loss = grad_loss.detach().to(torch.float32).contiguous()
        grad_image = torch.empty_like(image)
        height, width, channels = image.shape
        with torch.cuda.device(image.device):
            stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            native.check(native.lib().gs_l1_loss_backward(
                _ptr(image), height, width, channels, _ptr(target), target.shape[0],
                target.shape[1], _ptr(grad_loss), _ptr(grad_image), stream),
                "gs_l1_loss_backward")
        return grad_image, None


def l1_loss(image: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """``(image[:h, :w] - target).abs().mean()`` for a rendered ``image``
    [H, W, C] (padded to whole tiles) and ``target`` [h, w, C] covering its
    top-left corner, as a scalar device tensor; differentiable in ``image``
    (the target is data: a target that requires grad is refused)."""
    _check(image, target)
    if target.requires_grad:
        raise ValueError("l1_loss gives no gradient to the target")
    return _L1Loss.apply(image, target)
