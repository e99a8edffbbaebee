"""The fused L1 loss against torch's expression of it."""

import pytest
import torch

from gaussian_splats_b200.losses import l1_loss

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,crop", [((96, 136, 3), (90, 130)), ((1088, 1920, 3), (1080, 1920)),
                                        ((16, 16, 3), (16, 16))])
def test_l1_loss_matches_torch(shape, crop):
    g = torch.Generator(device="cuda").manual_seed(7)
    image = torch.rand(shape, device="cuda", generator=g)
    target = torch.rand((crop[0], crop[1], shape[2]), device="cuda", generator=g)
    target[::7, ::5] = image[:crop[0]:7, :crop[1]:5]  # exact ties: zero gradient there
    ours_in = image.clone().requires_grad_()
    ref_in = image.clone().requires_grad_()
    ours = l1_loss(ours_in, target)
    ref = (ref_in[:crop[0], :crop[1]] - target).abs().mean()
    torch.testing.assert_close(ours, ref, rtol=1e-6, atol=0)
    upstream = torch.tensor(0.37, device="cuda")
    (ours * upstream).backward()
    (ref * upstream).backward()
    assert torch.equal(ours_in.grad, ref_in.grad)  # torch's gradient values, bit for bit
    assert torch.count_nonzero(ours_in.grad[crop[0]:]) == 0


def test_l1_loss_refuses_target_gradients():
    image = torch.rand(8, 8, 3, device="cuda", requires_grad=True)
    with pytest.raises(ValueError, match="no gradient to the target"):
        l1_loss(image, torch.rand(8, 8, 3, device="cuda", requires_grad=True))
