"""render_dynamic_bank (the bank evaluated inside the projection kernel) against the reference's
_eval_dynamic_bank + dense render + loss (tests/golden/bank.npz)."""
import numpy as np
import pytest
import torch

from conftest import grad_close, load_golden
from dynaworld_b200.bank import DynamicGaussianBank, render_dynamic_bank
from dynaworld_b200.config import B200RendererConfig
from dynaworld_b200.losses import reconstruction_loss_per_image
from dynaworld_b200.renderer import render_b200_3dgs_batch
from gpu_helpers import DEV

pytestmark = pytest.mark.gpu

BANK = load_golden("bank")
BANK_KEYS = ("xyz0", "scales", "quats0", "opacities0", "rgbs", "A_mu", "A_rot", "A_alpha")
STATIC_KEYS = ("xyz", "scales", "quats", "opacities", "rgbs")


def case(name):
    return {k[len(name) + 1:]: torch.from_numpy(np.array(v)) for k, v in BANK.items() if k.startswith(name + "_")}


def leaves_of(t):
    bank = {k: t[f"bank_{k}"].to(DEV).requires_grad_(True) for k in BANK_KEYS}
    static = {k: t[f"static_{k}"].to(DEV).requires_grad_(True) for k in STATIC_KEYS} if "static_xyz" in t else None
    return bank, static


def render(t, bank, static, cfg=None):
    H, W = int(t["height"]), int(t["width"])
    return render_dynamic_bank(
        DynamicGaussianBank(**bank), t["times"].to(DEV), H, W, t["fx"].to(DEV), t["fy"].to(DEV), t["cx"].to(DEV),
        t["cy"].to(DEV), camera_to_world=t["camera_to_world"].to(DEV),
        static=None if static is None else tuple(static[k] for k in STATIC_KEYS),
        max_frequency=float(t["max_frequency"]), config=cfg)


@pytest.mark.parametrize("name", ["mixed", "odd"])
@pytest.mark.parametrize("batched", [False, True])
def test_bank_render_matches_reference(name, batched):
    t = case(name)
    bank, static = leaves_of(t)
    given = {k: (v[None] if batched else v) for k, v in bank.items()}  # the head's [1, G, ...] too
    image, alpha, depth = render(t, given, static)
    assert depth is None and alpha.shape == image[:, 0].shape
    assert (image.detach().cpu() - t["image"]).abs().max().item() <= 1e-4
    loss = reconstruction_loss_per_image(image, t["target"].to(DEV))
    torch.testing.assert_close(loss.detach().cpu(), t["loss"], rtol=1e-4, atol=2e-6)
    loss.sum().backward()
    leaves = {f"bank_{k}": v for k, v in bank.items()}
    if static is not None:
        leaves.update({f"static_{k}": v for k, v in static.items()})
    for k, v in leaves.items():
        ok, e, s = grad_close(v.grad.cpu(), t[f"grad_{k}"], 1e-3)
        assert ok, f"{name} {k}: {e:.3e} vs {s:.3e}"
    if name == "odd":  # opacities outside the logit clamp get no gradient
        assert (bank["opacities0"].grad[:15] == 0).all()


def test_zero_coefficients_render_the_base_frame():
    """With A = 0 every frame is the bank's base Gaussians (quaternion and opacity re-normalised
    through the identity rotation and logit/sigmoid): the activated render of those."""
    t = case("mixed")
    bank, _ = leaves_of(t)
    with torch.no_grad():
        for k in ("A_mu", "A_rot", "A_alpha"):
            bank[k].zero_()
        bank["opacities0"].clamp_(0.01, 0.99)
    image, _, _ = render(t, bank, None)
    K = image.shape[0]
    H, W = image.shape[-2:]
    base = render_b200_3dgs_batch(*(bank[k].detach()[None].expand(K, *bank[k].shape).contiguous()
                                    for k in ("xyz0", "scales", "quats0", "opacities0", "rgbs")), H, W,
                                  t["fx"].to(DEV), t["fy"].to(DEV), t["cx"].to(DEV), t["cy"].to(DEV),
                                  camera_to_world=t["camera_to_world"].to(DEV))
    assert (image.detach() - base).abs().max().item() <= 2e-5


def test_depth_output_and_segments():
    """Depth on and every backward segmentation: same image, gradients within 1e-4."""
    t = case("mixed")
    outs = []
    for seg in (1, 4):
        bank, static = leaves_of(t)
        image, alpha, depth = render(t, bank, static, B200RendererConfig(depth=True, backward_segments=seg))
        assert depth is not None and depth.shape == alpha.shape
        (reconstruction_loss_per_image(image, t["target"].to(DEV)).sum() + 1e-3 * depth.sum()).backward()
        outs.append((image.detach(), {k: v.grad for k, v in bank.items()}))
    assert torch.equal(outs[0][0], outs[1][0])
    for k in BANK_KEYS:
        ok, e, s = grad_close(outs[1][1][k], outs[0][1][k], 1e-4)
        assert ok, f"{k}: {e:.3e} vs {s:.3e}"


def test_bank_argument_errors():
    t = case("odd")
    bank, _ = leaves_of(t)
    with pytest.raises(NotImplementedError, match="decode times"):
        render_dynamic_bank(DynamicGaussianBank(**bank), t["times"].to(DEV).requires_grad_(True), 8, 8, 10.0, 10.0,
                            4.0, 4.0)
    wide = dict(bank, A_mu=torch.zeros(500, 17, 3, device=DEV), A_rot=torch.zeros(500, 17, 3, device=DEV),
                A_alpha=torch.zeros(500, 17, 1, device=DEV))
    with pytest.raises(ValueError, match="basis functions"):
        render_dynamic_bank(DynamicGaussianBank(**wide), t["times"].to(DEV), 8, 8, 10.0, 10.0, 4.0, 4.0)
    bad = dict(bank, A_rot=bank["A_rot"][:, :3])
    with pytest.raises(ValueError, match="A_rot"):
        render_dynamic_bank(DynamicGaussianBank(**bad), t["times"].to(DEV), 8, 8, 10.0, 10.0, 4.0, 4.0)
