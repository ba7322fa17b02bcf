"""Landmark-bank oracle (TEST INFRASTRUCTURE, see oracle/__init__.py).

Restates the decisions and the cache layout of the reference's v2 bank,
longctx/inference/landmark_cache_v2.py:
  _bank_D         :90-98    pairwise pose distance (numpy fp64)
  LandmarkCacheV2 :413-536  sink / recent window / always-admit bank
  _evict_index    :465-479  protect-earliest-n, most-redundant, later-born on ties
  _bank_insert    :481-495
  add_chunk       :498-536  (the optional env-var variants are off, as by default)
  _retrieve       :538-592  plain top-k by pose_dist, ascending indices
  write_into_cache :618-682 layout sink | recent (old -> new) | bank[R]
and pose_dist of longctx/inference/landmark_cache.py:24-31.  Chunks are
identified by their birth index; K/V bytes are reconstructed by the tests.
The budget split follows pipeline/causal_diffusion_inference_compressed.py:316-322.
"""
import math

import numpy as np


def pose_dist(a, b):
    """landmark_cache.py:24-31."""
    dxyz = float(np.linalg.norm(a[:3, 3] - b[:3, 3]))
    ya = math.degrees(math.atan2(a[0, 2], a[2, 2]))
    yb = math.degrees(math.atan2(b[0, 2], b[2, 2]))
    d = abs(ya - yb) % 360.0
    dyaw = min(d, 360.0 - d) / 60.0
    return math.sqrt(dxyz * dxyz + dyaw * dyaw)


def bank_D(poses):
    """landmark_cache_v2.py:90-98."""
    P = np.stack([np.asarray(p, dtype=np.float64) for p in poses])
    t = P[:, :3, 3]
    yaw = np.degrees(np.arctan2(P[:, 0, 2], P[:, 2, 2]))
    dt = np.linalg.norm(t[:, None, :] - t[None, :, :], axis=-1)
    dy = np.abs(yaw[:, None] - yaw[None, :]) % 360.0
    dy = np.minimum(dy, 360.0 - dy) / 60.0
    return np.sqrt(dt * dt + dy * dy)


def budget_split(budget_chunks, n_sink, recent_w, landmark_k):
    """compressed.py:316-322 -> (n_sink, eff_recent, n_landmark, bank_K) for mode 'b'."""
    eff_recent = min(recent_w, max(1, budget_chunks - n_sink - 1))
    n_landmark = max(1, budget_chunks - n_sink - eff_recent)
    bank_K = max(landmark_k, n_landmark)
    return n_sink, eff_recent, n_landmark, bank_K


class _Member:
    __slots__ = ("born", "pose", "protected")

    def __init__(self, born, pose):
        self.born = born
        self.pose = np.asarray(pose).copy()
        self.protected = False


class OracleBank:
    """Decision/layout restatement of LandmarkCacheV2 (mode 'a' or 'b')."""

    def __init__(self, n_sink=1, recent_w=5, K=30, retrieve_k=6, mode="b", protect_n=2):
        assert mode in ("a", "b")
        self.n_sink, self.recent_w, self.K = n_sink, recent_w, K
        self.retrieve_k, self.mode, self.protect_n = retrieve_k, mode, protect_n
        self.sink, self.recent, self.bank = [], [], []   # lists of born / _Member
        self.poses = {}
        self._n = 0
        self._admitted = 0
        self.events = []

    def _evict_index(self):
        n = len(self.bank)
        if n == 1:
            return 0
        D = bank_D([m.pose for m in self.bank])
        np.fill_diagonal(D, np.inf)
        nn = D.min(axis=1)
        cand = [i for i in range(n) if not self.bank[i].protected]
        if not cand:
            cand = list(range(n))
        return min(cand, key=lambda i: (nn[i], -self.bank[i].born))

    def _bank_insert(self, born):
        while len(self.bank) >= self.K:
            j = self._evict_index()
            victim = self.bank.pop(j)
            self.events.append(("evict", victim.born))
        m = _Member(born, self.poses[born])
        m.protected = self._admitted < self.protect_n
        self._admitted += 1
        self.bank.append(m)
        self.events.append(("add", born, len(self.bank)))

    def add_chunk(self, pose, pose_next=None):
        c = self._n
        self._n += 1
        self.poses[c] = np.asarray(pose).copy()
        if c < self.n_sink:
            self.sink.append(c)
        else:
            self.recent.append(c)
            while len(self.recent) > self.recent_w:
                self._bank_insert(self.recent.pop(0))
        return self._retrieve(pose_next if pose_next is not None else pose)

    def _retrieve(self, target):
        if not self.bank:
            return []
        if self.mode == "a":
            return list(range(len(self.bank)))
        ds = [pose_dist(target, m.pose) for m in self.bank]
        keep = [int(i) for i in np.argsort(ds) if np.isfinite(ds[i])]
        return sorted(keep[: self.retrieve_k])

    def layout(self, R):
        """Birth indices of the chunks write_into_cache puts at [0, tot): sink | recent | bank[R]."""
        return list(self.sink) + list(self.recent) + [self.bank[i].born for i in R]

    def bank_borns(self):
        return [m.born for m in self.bank]
