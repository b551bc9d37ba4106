"""The backward's bucketed chain rule (gsb_preprocess_bwd_range, used when a data-parallel
reducer is installed) on one GPU: a reducer that records the buckets instead of summing over
ranks must leave the gradients equal to the one-launch chain rule (up to the order of the
reverse blend's float atomics, which differs between any two runs), hand over every Gaussian's
rows exactly once, and return gradients that are views of one flat buffer."""
import pytest
import torch

from conftest import grad_close
from dynaworld_b200 import synthetic
from dynaworld_b200.distributed import shared_span
from dynaworld_b200.render import set_gradient_reducer
from gpu_helpers import render_raw

pytestmark = pytest.mark.gpu


class RecordingReducer:
    def __init__(self, buckets):
        self.buckets = buckets
        self.rows = []

    def active(self):
        return True

    def reduce(self, views):
        self.rows.append(views[0].shape[0])

    def finish(self):
        pass


@pytest.mark.parametrize("buckets", [1, 3, 7])
def test_bucketed_chain_rule_matches_one_launch(buckets):
    wl = synthetic.dynamic128(scale=1 / 16, image_scale=0.5, frames=4)
    ref = render_raw(wl)
    rec = RecordingReducer(buckets)
    set_gradient_reducer(rec)
    try:
        out = render_raw(wl)
    finally:
        set_gradient_reducer(None)
    assert sum(rec.rows) == wl.n_gaussians and len(rec.rows) == buckets
    for k in ("means", "log_scales", "quats", "opacity_logits", "sh", "velocity"):
        ok, err, scale = grad_close(out[f"grad_{k}"], ref[f"grad_{k}"], 1e-5)
        assert ok, f"{k}: {err:.3e} vs {scale:.3e}"


def test_gradients_are_views_of_one_buffer():
    from dynaworld_b200.renderer import render_b200
    from gpu_helpers import DEV, intrinsics_of

    wl = synthetic.static64(scale=0.25, image_scale=0.5)
    leaves = {k: getattr(wl, k).to(DEV).requires_grad_(True) for k in
              ("means", "log_scales", "quats", "opacity_logits", "sh")}
    image, _, _ = render_b200(leaves["means"], leaves["log_scales"], leaves["quats"], leaves["opacity_logits"],
                              leaves["sh"], intrinsics=intrinsics_of(wl), camera_to_world=wl.camera_to_world.to(DEV),
                              height=wl.height, width=wl.width)
    image.sum().backward()
    assert shared_span([v.grad for v in leaves.values()]) is not None
