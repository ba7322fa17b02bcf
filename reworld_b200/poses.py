"""Seeded synthetic camera trajectories for the rollout and bank benchmarks.

There is no dataset on this path: the reference's evaluation trajectories are
keyboard/mouse sequences turned into c2w poses (utils/camera.py:766-843: yaw
about the world Y axis, then pitch about the camera's right axis, translation
in the world frame).  These generators produce float32 4x4 c2w poses with the
same composition from seeded random increments, in the style of the
reference's own bank self-test walk (longctx/inference/landmark_cache_v2.py:729-743).
"""
import math

import numpy as np


def _axis_angle(axis, angle):
    axis = np.asarray(axis, dtype=np.float64)
    n = np.linalg.norm(axis)
    if n == 0.0 or angle == 0.0:
        return np.eye(3)
    x, y, z = axis / n
    c, s = math.cos(angle), math.sin(angle)
    C = 1.0 - c
    return np.array([[c + x * x * C, x * y * C - z * s, x * z * C + y * s],
                     [y * x * C + z * s, c + y * y * C, y * z * C - x * s],
                     [z * x * C - y * s, z * y * C + x * s, c + z * z * C]])


def random_walk(n, seed=0, step_t=0.1, step_deg=5.0, revisit_every=0, revisit_noise=0.01):
    """n float32 c2w poses: per step a translation N(0, step_t) per world axis and
    yaw/pitch increments N(0, step_deg) degrees.  With revisit_every = r > 0 the
    pose of every r-th chunk c replays the pose of chunk c - r plus
    N(0, revisit_noise) translation noise (a trajectory that returns to earlier
    places)."""
    rng = np.random.default_rng(seed)
    R = np.eye(3)
    t = np.zeros(3)
    out = []
    for c in range(n):
        dt = rng.normal(0.0, step_t, 3)
        dyaw, dpitch = np.radians(rng.normal(0.0, step_deg, 2))
        R = _axis_angle([0.0, 1.0, 0.0], dyaw) @ R
        R = _axis_angle(R[:, 0], dpitch) @ R
        u, _, vt = np.linalg.svd(R)
        R = u @ vt
        t = t + dt
        p = np.eye(4, dtype=np.float32)
        p[:3, :3] = R
        p[:3, 3] = t
        if revisit_every and c >= revisit_every and c % revisit_every == 0:
            p = out[c - revisit_every].copy()
            p[:3, 3] += rng.normal(0.0, revisit_noise, 3).astype(np.float32)
            R = p[:3, :3].astype(np.float64)
            t = p[:3, 3].astype(np.float64)
        out.append(p)
    return out


def yaw_walk(n, seed=0, step_t=0.35, step_yaw_deg=25.0):
    """Yaw-only walk with float32 poses (translation N(0, step_t), yaw N(0, step_yaw_deg))."""
    rng = np.random.default_rng(seed)
    poses, t, yaw = [], np.zeros(3), 0.0
    for _ in range(n):
        t = t + rng.normal(0.0, step_t, 3)
        yaw = (yaw + rng.normal(0.0, step_yaw_deg)) % 360.0
        r = math.radians(yaw)
        p = np.eye(4, dtype=np.float32)
        c, s = math.cos(r), math.sin(r)
        p[0, 0], p[0, 2], p[2, 0], p[2, 2] = c, s, -s, c
        p[:3, 3] = t
        poses.append(p)
    return poses
