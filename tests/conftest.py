import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libgsb200.so")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


class Golden(dict):
    """npz fixture as a dict of numpy arrays, with torch helpers."""

    def t(self, key, device="cpu", dtype=None):
        v = torch.from_numpy(np.array(self[key]))
        if dtype is not None:
            v = v.to(dtype)
        return v.to(device)

    def workload(self):
        from dynaworld_b200.synthetic import Workload

        vel = self.t("velocity") if "velocity" in self else None
        return Workload(
            name="golden", means=self.t("means"), log_scales=self.t("log_scales"), quats=self.t("quats"),
            opacity_logits=self.t("opacity_logits"), sh=self.t("sh"), velocity=vel, fx=self.t("fx"),
            fy=self.t("fy"), cx=self.t("cx"), cy=self.t("cy"), camera_to_world=self.t("camera_to_world"),
            times=self.t("times"), views_per_set=int(self["views_per_set"]), height=int(self["height"]),
            width=int(self["width"]), target=self.t("target"),
        )


def load_golden(name: str) -> Golden:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return Golden({k: z[k] for k in z.files})


GOLDEN_CASES = ["static64", "dynamic128_small", "multiview384_small", "clips256_small", "edge"]


@pytest.fixture(params=GOLDEN_CASES)
def golden_case(request):
    return request.param, load_golden(request.param)


# Per-element gradient tolerance: |g - g_ref| <= GRAD_RTOL * |g_ref| + GRAD_ATOL_FRAC * max|g_ref|.
# The floor is one part in 1e4 of the tensor's largest entry (ten times below the 1e-3-of-scale
# bar): an entry that is a sum of per-pixel terms cancelling far below the tensor's scale (a mean
# gradient over a nearly symmetric footprint, say) carries the float32 rounding of its terms, not
# of its value, in the reference's own float32 computation as in this one.
GRAD_RTOL = 1e-3
GRAD_ATOL_FRAC = 1e-4


def grad_close_elementwise(got: torch.Tensor, ref: torch.Tensor, rtol: float = GRAD_RTOL,
                           atol_frac: float = GRAD_ATOL_FRAC):
    """Per-element gradient parity: every |got - ref| <= rtol * |ref| + atol_frac * max |ref|.
    Returns (ok, worst excess ratio err / bound, the scale max |ref|)."""
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    scale = ref.abs().max().item()
    bound = rtol * ref.abs() + atol_frac * max(scale, 1e-30)
    ratio = ((got - ref).abs() / bound).max().item() if ref.numel() else 0.0
    return ratio <= 1.0, ratio, scale


def grad_close(got: torch.Tensor, ref: torch.Tensor, rel: float = 1e-3):
    """Gradient parity: max |got - ref| <= rel * max |ref| (the tensor's own scale)."""
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    return err <= rel * max(scale, 1e-30), err, scale
