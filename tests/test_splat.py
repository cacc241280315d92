"""splat_particles_2d (crates/burn_automata_kernels/src/splat.rs:30-93).

CPU: the oracle against the reference's known-answer test
(crates/burn_automata_kernels/src/lib.rs:405-418) and a direct Python
restatement on small cases.  GPU: the CUDA splat against the oracle (exp is
libm's expf on the host and a correctly rounded f64 exp on the device, hence
the tolerance), and device tensors against host buffers."""

import math

import numpy as np
import pytest

import oracle
from burn_automata_b200 import workloads
from burn_automata_b200.config import Splat2dConfig

f32 = np.float32


def splat_python(positions, colors, cfg):
    """splat.rs:30-93 line by line in f32 (small cases only)."""
    size = cfg.image_size
    out = np.zeros((size * size, 4), np.float32)
    sigma = f32(cfg.sigma)
    fsize = f32(size)
    span = f32(cfg.hi) - f32(cfg.lo)
    if cfg.normalize_color:
        sigma = sigma * fsize * f32(cfg.pixel_size) / span
    radius = int(max(f32(math.ceil(f32(5.0) * sigma)), f32(1.0)))
    norm_scale = (fsize * f32(cfg.pixel_size) / span) ** 2 if cfg.normalize_color else f32(1.0)
    norm_scale = f32(norm_scale)
    two_s2 = f32(2.0) * sigma * sigma
    for pos, color in zip(np.asarray(positions, np.float32), np.asarray(colors, np.float32)):
        px = (pos[0] - f32(cfg.lo)) / span * (fsize - f32(1.0))
        py = (pos[1] - f32(cfg.lo)) / span * (fsize - f32(1.0))
        if cfg.y_up:
            py = (fsize - f32(1.0)) - py
        bx, by = int(math.floor(px)), int(math.floor(py))
        fx, fy = px - f32(bx), py - f32(by)
        weights = []
        wsum = f32(0.0)
        for oy in range(-radius, radius + 1):
            for ox in range(-radius, radius + 1):
                x, y = bx + ox, by + oy
                if x < 0 or y < 0 or x >= size or y >= size:
                    continue
                dx, dy = f32(ox) - fx, f32(oy) - fy
                w = f32(math.exp(float(-(dx * dx + dy * dy) / two_s2)))
                weights.append((x, y, w))
                wsum = f32(wsum + w)
        denom = max(wsum, f32(1e-8)) if cfg.normalize_color else f32(1.0)
        for x, y, w in weights:
            w = w / denom * norm_scale
            p = out[y * size + x]
            p[0] = p[0] + color[0] * w
            p[1] = p[1] + color[1] * w
            p[2] = p[2] + color[2] * w
            p[3] = p[3] + w
    return out


def test_oracle_reference_kat():
    img = oracle.splat_particles_2d(np.zeros((1, 4), np.float32),
                                    np.array([[1.0, 0.0, 0.0]], np.float32),
                                    Splat2dConfig(image_size=8))
    assert img.shape == (64, 4) and (img[:, 3] > 0).any()


@pytest.mark.parametrize("cfg", [Splat2dConfig(image_size=16, pixel_size=2 / 16),
                                 Splat2dConfig(image_size=12, sigma=1.5, normalize_color=False,
                                               y_up=False)])
def test_oracle_matches_python_restatement(cfg):
    rng = np.random.default_rng(4)
    pos = np.zeros((40, 4), np.float32)
    pos[:, :2] = rng.uniform(-1.2, 1.2, (40, 2))
    col = rng.uniform(0, 1, (40, 3)).astype(np.float32)
    np.testing.assert_allclose(oracle.splat_particles_2d(pos, col, cfg),
                               splat_python(pos, col, cfg), rtol=1e-6, atol=1e-8)


def cases():
    rng = np.random.default_rng(11)
    w = workloads.make("cfg0", n=4096, steps=1)
    col = np.clip(w.states.reshape(-1, 16)[:, 13:16] + 0.5, 0, 1).astype(np.float32)
    out = np.zeros((300, 4), np.float32)
    out[:, :2] = rng.uniform(-3, 3, (300, 2))  # many outside the image
    return [
        ("kat", np.zeros((1, 4), np.float32), np.array([[1, 0, 0]], np.float32),
         Splat2dConfig(image_size=8)),
        ("cfg0_default", w.positions, col, Splat2dConfig()),
        ("cfg0_64", w.positions, col, Splat2dConfig(image_size=64)),
        ("raw_yup_off", w.positions[:1000], col[:1000],
         Splat2dConfig(image_size=40, sigma=1.5, normalize_color=False, y_up=False)),
        ("outside", out, rng.uniform(0, 1, (300, 3)).astype(np.float32),
         Splat2dConfig(image_size=48, pixel_size=2 / 48)),
        ("wide_sigma", w.positions[:64], col[:64],
         Splat2dConfig(image_size=24, sigma=8.0, pixel_size=2 / 24)),
        ("empty", np.zeros((0, 4), np.float32), np.zeros((0, 3), np.float32),
         Splat2dConfig(image_size=16)),
    ]


@pytest.mark.gpu
@pytest.mark.parametrize("case", cases(), ids=lambda c: c[0])
def test_gpu_splat_matches_oracle(case):
    import burn_automata_b200 as ba

    _, pos, col, cfg = case
    got = ba.splat_particles_2d(pos, col, cfg)
    want = oracle.splat_particles_2d(pos, col, cfg)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7)


@pytest.mark.gpu
def test_gpu_splat_device_tensors_match_host():
    import torch

    import burn_automata_b200 as ba

    _, pos, col, cfg = cases()[1]
    host = ba.splat_particles_2d(pos, col, cfg)
    dev = ba.splat_particles_2d(torch.from_numpy(pos).cuda(), torch.from_numpy(col).cuda(), cfg)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev.cpu().numpy(), host)
