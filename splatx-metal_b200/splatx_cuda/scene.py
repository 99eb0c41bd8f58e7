"""Seeded synthetic scenes with the shapes and value distributions of the benchmark configs.

No dataset is available (the reference benchmarks on Mip-NeRF 360 "garden"); these scenes stand in
for it with the distributions the benchmark configs state:
  cfg0  N=2,048 means U[-1,1]^3 + z in [2,6] before a 256x256 pinhole (fx=fy=300, c=128), SH deg 0
  cfg1/2 N=1,000,000 means N(0, 4 I), SH deg 3 (DC N(0,0.5), rest N(0,0.1)), one 1297x840 camera
        (fx=fy=1150) at distance 8 looking at the origin; cfg2's target is a render of a hidden
        seeded 200K-Gaussian scene.
Shared: log-scales N(-3,0.5), quats normalize(N(0,1)^4), opacity logits N(0,1).
Parameters are float32 in the reference's group layout: means[N,3], quats[N,4] (wxyz),
scales[N,3] (log), opacities[N] (logit), sh0[N,3], shN[N,K-1,3].
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Camera:
    viewmat: np.ndarray  # [16] row-major world->camera
    K: np.ndarray        # [9]
    width: int
    height: int


@dataclass
class Scene:
    means: np.ndarray
    quats: np.ndarray
    scales: np.ndarray
    opacities: np.ndarray
    sh0: np.ndarray
    shN: np.ndarray
    sh_degree: int

    @property
    def count(self) -> int:
        return self.means.shape[0]

    def groups(self):
        return [self.means, self.quats, self.scales, self.opacities, self.sh0, self.shN]


def _common(rng, n, sh_degree, dc_std, rest_std):
    K = (sh_degree + 1) ** 2
    q = rng.normal(size=(n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    scales = rng.normal(-3.0, 0.5, size=(n, 3)).astype(np.float32)
    opac = rng.normal(0.0, 1.0, size=n).astype(np.float32)
    sh0 = rng.normal(0.0, dc_std, size=(n, 3)).astype(np.float32)
    shN = rng.normal(0.0, rest_std, size=(n, K - 1, 3)).astype(np.float32)
    return q, scales, opac, sh0, shN


def small_scene(seed: int = 0, n: int = 2048, sh_degree: int = 0) -> tuple[Scene, Camera]:
    """cfg0-shaped scene and camera."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-1.0, 1.0, size=(n, 3)).astype(np.float32)
    means[:, 2] += rng.uniform(2.0, 6.0, size=n).astype(np.float32)
    q, s, o, sh0, shN = _common(rng, n, sh_degree, 0.5, 0.1)
    cam = Camera(np.eye(4, dtype=np.float32).ravel(),
                 np.array([300, 0, 128, 0, 300, 128, 0, 0, 1], np.float32), 256, 256)
    return Scene(means, q, s, o, sh0, shN.reshape(n, -1, 3), sh_degree), cam


def large_camera(distance: float = 8.0) -> Camera:
    W, H = 1297, 840
    vm = np.eye(4, dtype=np.float32)
    vm[2, 3] = distance  # camera on -z at `distance`, looking down +z at the origin
    K = np.array([1150, 0, W / 2, 0, 1150, H / 2, 0, 0, 1], np.float32)
    return Camera(vm.ravel(), K, W, H)


def orbit_camera(angle: float, distance: float = 8.0) -> Camera:
    """The cfg1/cfg2 camera carried around the scene's vertical axis by `angle` radians (angle 0
    is large_camera itself): the same distance, intrinsics and image, another side of the scene."""
    cam = large_camera(distance)
    c, s = np.cos(angle), np.sin(angle)
    rot_t = np.array([[c, 0.0, -s, 0.0], [0.0, 1.0, 0.0, 0.0], [s, 0.0, c, 0.0], [0.0, 0.0, 0.0, 1.0]])
    vm = cam.viewmat.reshape(4, 4).astype(np.float64) @ rot_t
    return Camera(vm.astype(np.float32).ravel(), cam.K, cam.width, cam.height)


def large_scene(seed: int = 0, n: int = 1_000_000, sh_degree: int = 3) -> tuple[Scene, Camera]:
    """cfg1/cfg2-shaped scene and camera."""
    rng = np.random.default_rng(seed)
    means = rng.normal(0.0, 2.0, size=(n, 3)).astype(np.float32)
    q, s, o, sh0, shN = _common(rng, n, sh_degree, 0.5, 0.1)
    return Scene(means, q, s, o, sh0, shN, sh_degree), large_camera()


def ring_camera(i: int, n_views: int, width: int = 1297, height: int = 840, seed: int = 0) -> Camera:
    """View i of a ring of cameras (radius 6-10, jittered elevation) looking at the origin."""
    rng = np.random.default_rng(seed * 100003 + i)
    ang = 2.0 * np.pi * i / n_views
    radius = rng.uniform(6.0, 10.0)
    elev = rng.uniform(-0.3, 0.3)
    c = np.array([radius * np.cos(ang) * np.cos(elev), radius * np.sin(elev),
                  radius * np.sin(ang) * np.cos(elev)])
    fwd = -c / np.linalg.norm(c)
    right = np.cross(np.array([0.0, 1.0, 0.0]), fwd)
    right /= np.linalg.norm(right)
    up = np.cross(fwd, right)
    R = np.stack([right, up, fwd])  # rows: camera axes in world coordinates
    t = -R @ c
    vm = np.eye(4)
    vm[:3, :3], vm[:3, 3] = R, t
    K = np.array([1150, 0, width / 2, 0, 1150, height / 2, 0, 0, 1], np.float32)
    return Camera(vm.astype(np.float32).ravel(), K, width, height)
