"""Fused optimizer step for training splats on the GPU.

The reference trains with ``torch.optim.Adam`` over one parameter group per
splat tensor (``training/train.py:111-118``: mean, rotation, scale, opacity,
color; ``eps=1e-15``), calls ``optimizer.step()`` after every backward
(``training/train.py:151``) and then perturbs the means with
``noise_splats`` (``training/utils.py:50-62``). :class:`FusedAdam` is that
optimizer with both steps done by one sm_100a kernel (``gs_adam_step``): each
parameter, gradient and moment element is read once and written once,
instead of ~30 elementwise kernels re-reading them.

It subclasses ``torch.optim.Adam`` and keeps its state layout (per parameter:
``step``, ``exp_avg``, ``exp_avg_sq``), so code that edits optimizer state
-- ``relocate_splats`` (``training/utils.py:147-210``) zeroing moments of
relocated splats or growing them when densifying -- works unchanged.
"""

from __future__ import annotations

import ctypes

import torch

from . import native

GROUP_NAMES = ("mean", "rotation", "scale", "opacity", "color")


class FusedAdam(torch.optim.Adam):
    """``torch.optim.Adam`` for a splat's five parameter tensors, one kernel
    per step.

    Build it the way the reference builds its optimizer: one group per
    tensor, each with a ``"name"`` from :data:`GROUP_NAMES` and one CUDA
    float32 contiguous parameter, e.g. ``FusedAdam([{"params": [s.mean],
    "name": "mean", "lr": 1.6e-4}, ...], eps=1e-15)``. Plain Adam only
    (no weight decay, amsgrad or maximize); anything else raises
    ``ValueError``. There is no CPU path.
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                         foreach=False)
        names = [group.get("name") for group in self.param_groups]
        if sorted(map(str, names)) != sorted(GROUP_NAMES):
            raise ValueError(f"FusedAdam needs one group per name in {GROUP_NAMES}, got {names}")
        for group in self.param_groups:
            if len(group["params"]) != 1:
                raise ValueError(f"group {group['name']!r} must hold exactly one tensor")
            if group["weight_decay"] or group["amsgrad"] or group["maximize"]:
                raise ValueError("FusedAdam supports plain Adam only (no weight decay, amsgrad "
                                 "or maximize)")
            if group["betas"] != self.param_groups[0]["betas"] or \
                    group["eps"] != self.param_groups[0]["eps"]:
                raise ValueError("FusedAdam needs the same betas and eps in every group")

    def _groups(self):
        by_name = {group["name"]: group for group in self.param_groups}
        return [by_name[name] for name in GROUP_NAMES]

    @torch.no_grad()
    def step(self, closure=None, noise=None):
        """One Adam step over the five groups (parameters without ``.grad``
        are skipped, as torch does). With ``noise=(noise_lr, position_lr)``
        the same kernel then adds noise_splats' position noise
        (``training/utils.py:50-62``) to the updated means, drawing its
        normal samples with ``torch.randn_like(mean)`` as the reference does."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        groups = self._groups()
        params = [group["params"][0] for group in groups]
        mean = params[0]
        n = mean.shape[0]
        for name, p in zip(GROUP_NAMES, params):
            if not (p.is_cuda and p.dtype == torch.float32 and p.is_contiguous()):
                raise RuntimeError(f"FusedAdam: {name} must be a contiguous CUDA float32 tensor "
                                   "(there is no CPU path)")
            if p.shape[0] != n or p.device != mean.device:
                raise RuntimeError(f"FusedAdam: {name} has {p.shape[0]} rows on {p.device}, "
                                   f"mean has {n} on {mean.device}")
        color = params[4]
        if color.dim() != 3 or color.shape[2] != 3:
            raise RuntimeError(f"FusedAdam: color must be [N, K, 3], got {tuple(color.shape)}")
        steps, grads = [], []
        for p in params:
            state = self.state[p]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0, dtype=torch.float32)
                state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            if p.grad is not None:
                if p.grad.is_sparse:
                    raise RuntimeError("FusedAdam does not support sparse gradients")
                state["step"] += 1
                grads.append(p.grad.contiguous())
            else:
                grads.append(None)
            steps.append(max(1.0, float(state["step"])))
        if all(g is None for g in grads) and noise is None:
            return loss
        beta1, beta2 = groups[0]["betas"]
        noise_lr, position_lr = noise if noise is not None else (0.0, 0.0)
        hyper = native.adam_params(steps, [float(g["lr"]) for g in groups], (beta1, beta2),
                                   groups[0]["eps"], noise_lr, position_lr)
        randn = torch.randn_like(mean) if noise is not None else None

        def arrays(tensors):
            return native.SplatArrays(*(t.data_ptr() if t is not None else None
                                        for t in tensors))

        sets = (arrays(params), arrays(grads),
                arrays([self.state[p]["exp_avg"] for p in params]),
                arrays([self.state[p]["exp_avg_sq"] for p in params]))
        with torch.cuda.device(mean.device):
            stream = ctypes.c_void_p(torch.cuda.current_stream(mean.device).cuda_stream)
            native.check(native.lib().gs_adam_step(
                n, color.shape[1], *(ctypes.byref(s) for s in sets), ctypes.byref(hyper),
                ctypes.c_void_p(randn.data_ptr() if randn is not None else None), stream),
                "gs_adam_step")
        return loss
