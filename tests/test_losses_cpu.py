"""Host checks of the fused L1 loss (no CPU path, shapes, target gradients)."""

import pytest
import torch

from gaussian_splats_b200.losses import l1_loss


def test_l1_loss_has_no_cpu_path():
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        l1_loss(torch.zeros(8, 8, 3), torch.zeros(8, 8, 3))


def test_l1_loss_checks_shapes():
    from gaussian_splats_b200 import losses

    class Fake:  # shape-only stand-ins for device tensors
        is_cuda = True
        device = "cuda:0"
        requires_grad = False

        def __init__(self, *shape):
            self.shape = shape

        def dim(self):
            return len(self.shape)

    with pytest.raises(ValueError, match="larger than the image"):
        losses._check(Fake(8, 8, 3), Fake(9, 8, 3))
    with pytest.raises(ValueError, match="expected"):
        losses._check(Fake(8, 8, 3), Fake(8, 8, 4))
