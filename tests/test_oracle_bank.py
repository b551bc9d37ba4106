"""The oracle's dynamic-bank evaluation, render, loss and gradients against the reference's own
(tests/golden/bank.npz, made by tests/golden/make_golden_bank.py), and the product's temporal
basis against the oracle's (CPU only)."""
import numpy as np
import pytest
import torch

from conftest import grad_close, load_golden
from dynaworld_b200.bank import temporal_basis
from oracle import bank_oracle as bo
from oracle import splat_oracle as so

BANK = load_golden("bank")
BANK_KEYS = ("xyz0", "scales", "quats0", "opacities0", "rgbs", "A_mu", "A_rot", "A_alpha")
STATIC_KEYS = ("xyz", "scales", "quats", "opacities", "rgbs")


def case(name):
    return {k[len(name) + 1:]: torch.from_numpy(np.array(v)) for k, v in BANK.items() if k.startswith(name + "_")}


@pytest.mark.parametrize("M", [1, 2, 5, 8, 16])
def test_temporal_basis_matches_oracle(M):
    t = torch.linspace(0.0, 1.0, 11)
    got = temporal_basis(t, M, 8.0).double()
    ref = bo.temporal_basis(t.double(), M, 8.0)
    assert got.shape == (11, M)
    assert (got - ref).abs().max().item() <= 2e-6


def test_temporal_basis_rejects_bad_arguments():
    with pytest.raises(ValueError, match="basis_count"):
        temporal_basis(torch.zeros(2), 0, 8.0)
    with pytest.raises(ValueError, match="max_frequency"):
        temporal_basis(torch.zeros(2), 4, 0.0)


@pytest.mark.parametrize("name", ["mixed", "odd"])
def test_bank_frames_match_reference(name):
    t = case(name)
    bank = {k: t[f"bank_{k}"].double() for k in BANK_KEYS}
    static = {k: t[f"static_{k}"].double() for k in STATIC_KEYS} if "static_xyz" in t else None
    xyz, _s, quats, opac, _c = bo.frames(bank, t["times"].double(), float(t["max_frequency"]), static)
    assert (xyz.float() - t["frame_xyz"]).abs().max().item() <= 2e-6
    assert (quats.float() - t["frame_quats"]).abs().max().item() <= 2e-6
    assert (opac.float() - t["frame_opacities"]).abs().max().item() <= 2e-6


@pytest.mark.parametrize("name", ["mixed", "odd"])
def test_bank_render_and_gradients_match_reference(name):
    t = case(name)
    H, W = int(t["height"]), int(t["width"])
    bank = {k: t[f"bank_{k}"].double().requires_grad_(True) for k in BANK_KEYS}
    static = ({k: t[f"static_{k}"].double().requires_grad_(True) for k in STATIC_KEYS}
              if "static_xyz" in t else None)
    xyz, scales, quats, opac, rgbs = bo.frames(bank, t["times"].double(), float(t["max_frequency"]), static)
    key = so.camera_depth_fp32(t["frame_xyz"], t["camera_to_world"])  # the reference's float32 depth order
    img, _, _ = so.render_dense(xyz, scales, quats, opac, rgbs, H, W, t["fx"].double(), t["fy"].double(),
                                t["cx"].double(), t["cy"].double(), t["camera_to_world"].double(), sort_key=key)
    assert (img.float() - t["image"]).abs().max().item() <= 1e-5
    loss = so.reconstruction_loss_per_image(img, t["target"].double())
    torch.testing.assert_close(loss.float(), t["loss"], rtol=1e-5, atol=1e-7)
    loss.sum().backward()
    leaves = {f"bank_{k}": v for k, v in bank.items()}
    if static is not None:
        leaves.update({f"static_{k}": v for k, v in static.items()})
    for k, v in leaves.items():
        ok, e, s = grad_close(v.grad, t[f"grad_{k}"], 1e-3)
        assert ok, f"{name} {k}: {e:.3e} vs {s:.3e}"
    if name == "odd":  # opacities outside the logit clamp get no gradient
        assert (bank["opacities0"].grad[:15] == 0).all()
