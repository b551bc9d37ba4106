"""Gradient checks that account for the clamps' kinks.

The reference's image is clamp(sum w c + (1 - clamp(sum w, 0, 1)) bg, 0, 1) (dense.py:232-233,
tiled.py:191-198).  torch passes a clamp's gradient when its input lies inside [0, 1] and blocks it
outside, so at a pixel whose weight sum (or pre-clamp colour) lies within float32 rounding of 0 or
1 the gradient jumps with the last bit of that sum: two correct float32 evaluations may land on
different sides.  Golden scenes have a few such pixels (clips256_small: two pixels whose weight sum
is within 3e-7 of 1).  A gradient entry that misses the per-element bound against the reference
passes here only if every gradient tensor meets the bound against the float64 oracle evaluated
with one choice of sides at the kink pixels (|value - bound| <= KINK_TOL, chosen pixel by pixel),
so the difference is shown to be that choice and nothing else.
"""
from __future__ import annotations

import torch

from conftest import GRAD_ATOL_FRAC, GRAD_RTOL
from oracle import splat_oracle as so
from oracle import tiled_oracle as to

KINK_TOL = 4e-6  # float32 weight sums over long lists carry a few 1e-7 of rounding
RAW = ("means", "log_scales", "quats", "opacity_logits", "sh")


def _excess(got, ref):
    """(worst ratio of |got - ref| to the per-element bound, summed excess over the bound)."""
    got, ref = got.detach().double().cpu(), ref.detach().double().cpu()
    scale = ref.abs().max().item()
    r = (got - ref).abs() / (GRAD_RTOL * ref.abs() + GRAD_ATOL_FRAC * max(scale, 1e-30))
    return r.max().item(), (r - 1.0).clamp_min(0.0).sum().item()


def _ratio(got, ref):
    return _excess(got, ref)[0]


def _oracle(wl, tiled_tile, flip_w=None, flip_i=None):
    """float64 oracle render + loss; returns (raw-parameter gradients, weight sums, pre-clamp image)."""
    leaves = {k: getattr(wl, k).double().requires_grad_(True) for k in RAW}
    vel = wl.velocity.double().requires_grad_(True) if wl.velocity is not None else None
    raw = so.RawGaussians(*(leaves[k] for k in RAW), vel)
    m, s, q, o, rgb = so.activate(raw, wl.times.double(), wl.camera_to_world, wl.views_per_set)
    if tiled_tile is None:
        key = so.camera_depth_fp32(m.float(), wl.camera_to_world)
        img, wsum, _d, pre = so.render_dense(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy,
                                             wl.camera_to_world, sort_key=key, flip_wsum=flip_w, flip_image=flip_i,
                                             return_pre=True)
    else:
        outs = [to.render_tiled_view(m[b], s[b], q[b], o[b], rgb[b], wl.height, wl.width, wl.fx[b], wl.fy[b],
                                     wl.cx[b], wl.cy[b], wl.camera_to_world[b], tile_size=tiled_tile,
                                     flip_wsum=None if flip_w is None else flip_w[b],
                                     flip_image=None if flip_i is None else flip_i[b], return_pre=True)
                for b in range(wl.n_views)]
        img = torch.stack([x[0] for x in outs])
        wsum = torch.stack([x[1] for x in outs])
        pre = torch.stack([x[2] for x in outs])
    so.reconstruction_loss_per_image(img, wl.target.double()).sum().backward()
    grads = {k: v.grad for k, v in leaves.items()}
    if vel is not None:
        grads["velocity"] = vel.grad
    return grads, wsum.detach(), pre.detach()


NEAR_PX = 12  # pixels from a Gaussian's projected centre within which a kink is considered


def _centres_of_misses(wl, got, ref):
    """(view, x, y) projected centres of the Gaussians with an entry that misses the bound."""
    S, G = wl.n_sets, wl.n_gaussians
    miss = torch.zeros(S * G, dtype=torch.bool)
    for k in ref:
        g_, r_ = got[k].detach().double().cpu(), ref[k].detach().double().cpu()
        scale = r_.abs().max().item()
        bad = (g_ - r_).abs() > GRAD_RTOL * r_.abs() + GRAD_ATOL_FRAC * max(scale, 1e-30)
        miss |= bad.reshape(S * G, -1).any(1)
    out = []
    for pg in torch.nonzero(miss).flatten().tolist():
        s_, g = divmod(pg, G)
        for b in range(s_ * wl.views_per_set, min((s_ + 1) * wl.views_per_set, wl.n_views)):
            t = float(wl.times[b])
            mean = wl.means[s_, g].double() + (t * wl.velocity[s_, g].double() if wl.velocity is not None else 0.0)
            c2w = wl.camera_to_world[b].double()
            d = (mean - c2w[:3, 3]) @ c2w[:3, :3]
            if d[2] > 1e-4:
                out.append((b, float(wl.fx[b] * d[0] / d[2] + wl.cx[b]), float(wl.fy[b] * d[1] / d[2] + wl.cy[b])))
    return out


def check_gradients(wl, got: dict, ref: dict, tiled_tile: int | None = None):
    """got / ref: raw-parameter gradients by name (GPU / reference fixture).  Raises AssertionError
    unless every tensor meets the per-element bound against the reference, or the tensors meet it
    against the oracle on one choice of sides at the scene's kink pixels."""
    ratios = {k: _ratio(got[k], ref[k]) for k in ref}
    if max(ratios.values()) <= 1.0:
        return
    _, wsum, pre = _oracle(wl, tiled_tile)
    kw = (wsum - 1.0).abs() <= KINK_TOL
    ki = (((pre - 1.0).abs() <= KINK_TOL) | (pre.abs() <= KINK_TOL)) & (wsum.unsqueeze(1) > 0)
    sites = [("w", tuple(i)) for i in kw.nonzero().tolist()] + [("i", tuple(i)) for i in ki.nonzero().tolist()]
    worst = {k: r for k, r in ratios.items() if r > 1.0}
    # only kinks near a Gaussian whose gradient misses the bound can explain it
    near = _centres_of_misses(wl, got, ref)
    sites = [(kind, idx) for kind, idx in sites
             if any(b == idx[0] and abs(y - idx[-2]) <= NEAR_PX and abs(x - idx[-1]) <= NEAR_PX for b, x, y in near)]
    assert sites, f"per-element bound missed with no kink pixel near the entries that miss it: {worst}"

    def score(flips):
        fw, fi = torch.zeros_like(kw), torch.zeros_like(ki)
        for kind, idx in flips:
            (fw if kind == "w" else fi)[idx] = True
        grads, _, _ = _oracle(wl, tiled_tile, fw, fi)
        ex = [_excess(got[k], grads[k]) for k in ref]
        return max(e[0] for e in ex), sum(e[1] for e in ex)

    # the sides are chosen site by site (kinks far apart touch different Gaussians): a flip is kept
    # when it lowers the summed excess, until every entry meets the bound
    chosen: set = set()
    cur = score(chosen)
    improved = True
    while cur[0] > 1.0 and improved:
        improved = False
        for site in sites:
            if site in chosen:
                continue
            trial = score(chosen | {site})
            if trial[1] < cur[1]:
                chosen, cur, improved = chosen | {site}, trial, True
                if cur[0] <= 1.0:
                    break
    assert cur[0] <= 1.0, (f"per-element bound missed ({worst}); against the oracle with {len(chosen)} of "
                           f"{len(sites)} kink pixels flipped: {cur[0]:.2f}")
