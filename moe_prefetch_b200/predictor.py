"""The predictor hook: MOEP v3 expert predictors, read and scored on the host.

``MoePredictor`` mirrors the reference's ``moe_predictor`` (cpp/moe-predictor.h
:38-106): ``load``, ``has_layer``, ``score``, ``top_k_ids``, ``update``,
``save``.  The model is per-layer ridge over multi-hot blocks
(prev / cur / below / self_prev, each n_expert wide): the score is the
layer's bias plus the weight rows the ids select, z-scored, plus the repeat
prior on the `prev` ids.  Scores are formed in fp32 with sequential
accumulation in the same order as the C++ (row adds in id order, mean and
variance as running sums), so they agree with it to rounding.

``ExpertPredictor`` is the PCA + ridge prototype of src/predictor.py:26-93.
"""
import math
import struct

import numpy as np

BLOCK_PCA, BLOCK_PREV, BLOCK_CUR, BLOCK_BELOW, BLOCK_SELF_PREV = 0, 1, 2, 3, 4
MAGIC = b"MOEP"
VERSION = 3


class MoepError(ValueError):
    pass


class MoePredictor:
    def __init__(self):
        self.n_expert = self.n_layers = self.feat_dim = self.top_k = 0
        self.d_model = self.n_comp = 0
        self.has_pca = False
        self.off = {BLOCK_PREV: -1, BLOCK_CUR: -1, BLOCK_BELOW: -1, BLOCK_SELF_PREV: -1,
                    BLOCK_PCA: -1}
        self.mean = self.comp = self.scale = None
        self.layer_of = np.zeros(0, np.int32)
        self.index_of = np.zeros(0, np.int32)
        self.prior = np.zeros(0, np.float32)
        self.bias = np.zeros((0, 0), np.float32)
        self.w = np.zeros((0, 0, 0), np.float32)

    # -- file format (cpp/moe-predictor.cpp:21-155, :320-362) ------------------
    @classmethod
    def load(cls, path):
        with open(path, "rb") as f:
            data = f.read()
        p = cls()
        if data[:4] != MAGIC:
            raise MoepError(f"{path}: not a MOEP file")
        pos = 4

        def u32():
            nonlocal pos
            if pos + 4 > len(data):
                raise MoepError(f"{path}: truncated header")
            v = struct.unpack_from("<I", data, pos)[0]
            pos += 4
            return v

        ver = u32()
        p.d_model, p.n_comp, p.n_expert, p.n_layers, p.top_k, p.feat_dim = (u32() for _ in range(6))
        n_present, n_blocks, pca_flag, _reserved = u32(), u32(), u32(), u32()
        if ver != VERSION:
            raise MoepError(f"{path}: version {ver}, expected 3")
        p.has_pca = pca_flag != 0
        expect = 0
        for i in range(n_blocks):
            kind, off, size = u32(), u32(), u32()
            if off != expect:
                raise MoepError(f"{path}: block {i} starts at {off}, expected {expect}")
            expect += size
            if kind == BLOCK_PCA:
                if size != p.n_comp:
                    raise MoepError(f"{path}: PCA block size != n_comp")
            elif kind in (BLOCK_PREV, BLOCK_CUR, BLOCK_BELOW, BLOCK_SELF_PREV):
                if size != p.n_expert:
                    raise MoepError(f"{path}: block size != n_expert")
            else:
                raise MoepError(f"{path}: unknown feature block kind {kind}")
            p.off[kind] = off
        if expect != p.feat_dim:
            raise MoepError(f"{path}: blocks cover {expect} columns, feat_dim is {p.feat_dim}")
        if p.has_pca != (p.off[BLOCK_PCA] >= 0):
            raise MoepError(f"{path}: has_pca disagrees with the block table")

        def f32(n, what):
            nonlocal pos
            if pos + 4 * n > len(data):
                raise MoepError(f"{path}: truncated {what}")
            a = np.frombuffer(data, np.float32, n, pos).copy()
            pos += 4 * n
            return a

        if p.has_pca:
            p.mean = f32(p.d_model, "PCA block")
            p.comp = f32(p.d_model * p.n_comp, "PCA block").reshape(p.d_model, p.n_comp)
            p.scale = f32(p.n_comp, "PCA block")
        if pos + 4 * n_present > len(data):
            raise MoepError(f"{path}: truncated layer table")
        p.layer_of = np.frombuffer(data, np.int32, n_present, pos).copy()
        pos += 4 * n_present
        p.prior = f32(n_present, "layer table")
        p.bias = f32(n_present * p.n_expert, "layer table").reshape(n_present, p.n_expert)
        need = n_present * p.feat_dim * p.n_expert
        if pos + 4 * need > len(data):
            raise MoepError(f"{path}: truncated weights (wanted {4 * need} bytes)")
        p.w = f32(need, "weights").reshape(n_present, p.feat_dim, p.n_expert)
        if pos != len(data):
            raise MoepError(f"{path}: trailing bytes after the weights")
        p.index_of = np.full(p.n_layers, -1, np.int32)
        for i, il in enumerate(p.layer_of):
            if il < 0 or il >= p.n_layers:
                raise MoepError(f"{path}: layer index {il} out of range")
            p.index_of[il] = i
        return p

    def save(self, path):
        if self.has_pca:
            raise MoepError("refusing to save a predictor with a PCA block")
        blocks = sorted((off, kind) for kind, off in self.off.items()
                        if kind != BLOCK_PCA and off >= 0)
        # header: version, d_model, n_comp, n_expert, n_layers, top_k, feat_dim,
        #         n_present, n_blocks, pca_flag (0), reserved (0)
        out = [MAGIC, struct.pack("<11I", VERSION, self.d_model, self.n_comp, self.n_expert,
                                  self.n_layers, self.top_k, self.feat_dim, len(self.layer_of),
                                  len(blocks), 0, 0)]
        for off, kind in blocks:
            out.append(struct.pack("<3I", kind, off, self.n_expert))
        out += [self.layer_of.astype("<i4").tobytes(), self.prior.astype("<f4").tobytes(),
                self.bias.astype("<f4").tobytes(), self.w.astype("<f4").tobytes()]
        with open(path, "wb") as f:
            f.write(b"".join(out))

    # -- inference (cpp/moe-predictor.cpp:165-240) -----------------------------
    def has_layer(self, il):
        return 0 <= il < len(self.index_of) and self.index_of[il] >= 0

    def score(self, il, prev=(), cur=(), below=(), self_prev=()):
        slot = int(self.index_of[il])
        E = self.n_expert
        W = self.w[slot]
        out = self.bias[slot].copy()
        for ids, kind in ((prev, BLOCK_PREV), (cur, BLOCK_CUR), (below, BLOCK_BELOW),
                          (self_prev, BLOCK_SELF_PREV)):
            off = self.off[kind]
            if off < 0:
                continue
            for e in ids:
                e = int(e)
                if 0 <= e < E:
                    out += W[off + e]
        mu = np.float32(np.cumsum(out, dtype=np.float32)[-1]) / np.float32(E)
        d = out - mu
        var = np.cumsum(d * d, dtype=np.float32)[-1]
        sd = np.float32(math.sqrt(np.float32(var / np.float32(E)))) + np.float32(1e-9)
        out = ((out - mu) / sd).astype(np.float32)
        pw = self.prior[slot]
        if pw != 0.0:
            for e in prev:
                e = int(e)
                if 0 <= e < E:
                    out[e] += pw
        return out

    @staticmethod
    def top_k_ids(scores, k):
        """Best first, ties to the lower id (cpp/moe-predictor.cpp:226-240)."""
        s = np.asarray(scores)
        k = min(k, len(s))
        order = np.lexsort((np.arange(len(s)), -s.astype(np.float64)))
        return order[:k].astype(np.int32)

    def update(self, il, truth, lr, prev=(), cur=(), below=(), self_prev=()):
        """One logistic-SGD step (cpp/moe-predictor.cpp:243-311); returns the
        recall@8 of the prediction before the update."""
        if not self.has_layer(il) or len(truth) == 0:
            return 0.0
        slot = int(self.index_of[il])
        E = self.n_expert
        s = self.score(il, prev, cur, below, self_prev)
        y = np.zeros(E, np.uint8)
        for e in truth:
            if 0 <= int(e) < E:
                y[int(e)] = 1
        top = self.top_k_ids(s, 8)
        hit = float(np.float32(sum(int(y[t]) for t in top)) / np.float32(len(truth)))
        p = (np.float32(1.0) / (np.float32(1.0) + np.exp(-s).astype(np.float32))).astype(np.float32)
        g = ((p - y.astype(np.float32)) * np.float32(lr)).astype(np.float32)
        W = self.w[slot]
        for ids, kind in ((prev, BLOCK_PREV), (cur, BLOCK_CUR), (below, BLOCK_BELOW),
                          (self_prev, BLOCK_SELF_PREV)):
            off = self.off[kind]
            if off < 0:
                continue
            for e in ids:
                e = int(e)
                if 0 <= e < E:
                    W[off + e] -= g
        self.bias[slot] -= g
        return hit


class ExpertPredictor:
    """Per-layer ridge probes over a shared PCA basis (src/predictor.py:26-93)."""

    def __init__(self, mean, comp, scale, weights):
        self.mean = mean
        self.comp = comp
        self.scale = scale
        self.weights = weights

    @classmethod
    def fit(cls, H, E, pairs, train_mask, n_comp=256, lam=100.0):
        src, _dst = pairs
        rows = np.unique(src[train_mask])
        mean = H[rows].mean(0)
        Xc = H[rows] - mean
        cov = (Xc.T @ Xc) / max(len(Xc) - 1, 1)
        _w, V = np.linalg.eigh(cov.astype(np.float64))
        comp = V[:, ::-1][:, :n_comp].astype(np.float32)
        proj = (H[rows] - mean) @ comp
        scale = proj.std(0) + 1e-6
        return mean, comp, scale

    @classmethod
    def fit_layer(cls, X, Y, lam=100.0):
        G = X.T @ X + lam * np.eye(X.shape[1], dtype=np.float32)
        return np.linalg.solve(G, X.T @ Y).astype(np.float32)

    def project(self, h):
        return ((h - self.mean) @ self.comp) / self.scale

    def top_p(self, layer, h_proj, p=8):
        W = self.weights.get(layer)
        if W is None:
            return np.empty(0, dtype=np.int64)
        s = h_proj @ W
        return np.argpartition(-s, p)[:p]

    def scores(self, layer, h_proj):
        W = self.weights.get(layer)
        return None if W is None else h_proj @ W

    def save(self, path):
        np.savez_compressed(path, mean=self.mean, comp=self.comp, scale=self.scale,
                            layers=np.array(sorted(self.weights)),
                            stack=np.stack([self.weights[k] for k in sorted(self.weights)]))

    @classmethod
    def load(cls, path):
        d = np.load(path)
        weights = {int(k): w for k, w in zip(d["layers"], d["stack"])}
        return cls(d["mean"], d["comp"], d["scale"], weights)

    def n_params(self):
        return self.comp.size + sum(w.size for w in self.weights.values())
