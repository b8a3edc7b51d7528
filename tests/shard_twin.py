"""A numpy stand-in for the enx_shard_* device phases (enargeia_b200/csrc/k_shard.cu), with the
same inputs, outputs and buffer layouts, so the host protocol of enargeia_b200.vocab_shard can be
tested on CPU (lockstep, and across gloo ranks) without a GPU.  Test infrastructure only: the
product runs the CUDA phases."""

from __future__ import annotations

import numpy as np
import torch

f32 = np.float32
NONE = 0xFFFFFFFF


def _params(t: torch.Tensor) -> np.ndarray:
    return np.frombuffer(t.cpu().numpy().tobytes(), dtype=np.float32).reshape(-1, 4)


def _u32(t: torch.Tensor) -> np.ndarray:
    return t.numpy().view(np.uint32)


def _rank(n: int) -> int:
    d = n.bit_length() - 1
    return (2 * (n - (1 << d)) + 1) << (7 - d)


def _tree(lo, hi):
    L = np.zeros(256, f32)
    H = np.zeros(256, f32)
    mids = np.zeros(256, f32)
    thr = np.zeros(256, np.float64)
    L[1], H[1] = lo, hi
    for n in range(1, 256):
        mid = f32(f32(L[n] + H[n]) * f32(0.5))
        mids[n] = mid
        if n < 128:
            L[2 * n], H[2 * n] = L[n], mid
            L[2 * n + 1], H[2 * n + 1] = mid, H[n]
    for n in range(1, 256):
        thr[_rank(n)] = float(mids[n])
    return mids, thr


def _fx62(p):
    return np.rint(np.asarray(p, np.float64) * 2.0 ** 62).astype(np.uint64)


def _gidx(u, row, rows, split):
    return ((u // split) * rows + row) * split + u % split


class NumpyPhases:
    def state(self, rows, device):
        return {"lohi": np.zeros((rows, 5, 2), f32), "garg": np.zeros(rows, np.uint32), "thr": np.zeros(rows)}

    @staticmethod
    def _spans(n, split):
        per = -(-n // split)
        return [(min(c * per, n), min(min(c * per, n) + per, n)) for c in range(split)]

    def prepare(self, logits, n, row_begin, rows, split, history, hstride, hist_len, params, cand):
        L = logits.numpy()
        P = _params(params)
        out = _u32(cand).reshape(rows, split, 4)
        for r in range(rows):
            T, _, rp, _ = P[r]
            if rp != f32(1.0) and history is not None:
                hl = int(hist_len[r]) if hist_len is not None else hstride
                ids = set(int(i) for i in _u32(history)[r, :hl] if row_begin <= int(i) < row_begin + n)
                for i in ids:
                    v = L[r, i - row_begin]
                    L[r, i - row_begin] = v / rp if v > 0 else v * rp
            for c, (b, e) in enumerate(self._spans(n, split)):
                seg = L[r, b:e]
                gv, gi, sv, si = f32(-1e30), NONE, f32(-1e30), NONE
                if e > b:
                    k = int(np.argmax(seg))
                    if seg[k] > gv:
                        gv, gi = seg[k], row_begin + b + k
                    if T > 0:
                        s = (seg / T).astype(f32)
                        k = int(np.argmax(s))
                        if s[k] > sv:
                            sv, si = s[k], row_begin + b + k
                out[r, c] = [np.array(gv, f32).view(np.uint32), gi, np.array(sv, f32).view(np.uint32), si]

    def probs(self, logits, n, rows, split, world, params, cand_all, state, probs, sums):
        P = _params(params)
        L = logits.numpy()
        C = _u32(cand_all).reshape(-1, 4)
        p = probs.numpy().reshape(rows, n)
        S = sums.numpy().reshape(rows, split)
        for r in range(rows):
            T = P[r, 0]
            if T <= 0:
                S[r] = 0.0
                continue
            bv, bi = f32(-1e30), NONE
            for u in range(world * split):
                c = C[_gidx(u, r, rows, split)]
                v = c[2:3].view(f32)[0]
                if v > bv or (v == bv and c[3] < bi):
                    bv, bi = v, int(c[3])
            state["garg"][r] = 0 if bi == NONE else bi
            state["lohi"][r, 0] = (0.0, 1.0)
            p[r] = np.exp((L[r] / T).astype(f32).astype(np.float64) - float(bv))
            for c, (b, e) in enumerate(self._spans(n, split)):
                S[r, c] = p[r, b:e].sum()

    def _walk(self, bucket_all, r, rows, units, split, lo, hi, top_p):
        mids, _ = _tree(lo, hi)
        B = bucket_all.numpy().view(np.uint64).reshape(-1, 256)
        tot = np.zeros(256, np.uint64)
        for u in range(units):
            tot += B[_gidx(u, r, rows, split)]
        suffix = np.cumsum(tot[::-1])[::-1]
        goal = _fx62(np.float64(top_p))
        n, l, h = 1, lo, hi
        for _ in range(8):
            if suffix[_rank(n)] < goal:
                h, n = mids[n], 2 * n
            else:
                l, n = mids[n], 2 * n + 1
        return l, h

    def _normalise(self, sum_all, p, r, rows, units, split):
        gs = 0.0
        for u in range(units):
            gs += float(sum_all.numpy()[_gidx(u, r, rows, split)])
        p[r] /= gs

    def buckets(self, n, rows, split, world, rnd, params, sum_all, prev, state, probs, bucket):
        P = _params(params)
        p = probs.numpy().reshape(rows, n)
        out = bucket.numpy().view(np.uint64).reshape(rows, split, 256)
        units = world * split
        for r in range(rows):
            T, top_p = P[r, 0], P[r, 1]
            out[r] = 0
            if T <= 0:
                continue
            if rnd == 0:
                self._normalise(sum_all, p, r, rows, units, split)
            if top_p >= 1:
                continue
            lo, hi = f32(0.0), f32(1.0)
            if rnd > 0:
                lo, hi = self._walk(prev, r, rows, units, split, *state["lohi"][r, rnd - 1], top_p)
                state["lohi"][r, rnd] = (lo, hi)
            _, thr = _tree(lo, hi)
            for c, (b, e) in enumerate(self._spans(n, split)):
                seg = p[r, b:e]
                k = np.searchsorted(thr[1:256], seg, side="right")
                np.add.at(out[r, c], k, _fx62(seg))

    def kept(self, n, rows, split, world, rounds, params, sum_all, last, state, probs, kept):
        P = _params(params)
        p = probs.numpy().reshape(rows, n)
        K = kept.numpy().reshape(rows, split)
        units = world * split
        for r in range(rows):
            T, top_p = P[r, 0], P[r, 1]
            if T <= 0:
                K[r] = 0.0
                continue
            if rounds == 0:
                self._normalise(sum_all, p, r, rows, units, split)
            thr = 0.0
            if top_p < 1 and rounds > 0:
                thr = float(self._walk(last, r, rows, units, split, *state["lohi"][r, rounds - 1], top_p)[0])
            state["thr"][r] = thr
            for c, (b, e) in enumerate(self._spans(n, split)):
                seg = p[r, b:e]
                K[r, c] = seg[seg >= thr].sum()

    def pick(self, n, row_begin, rows, split, world, rank, params, kept_all, state, probs, pick):
        P = _params(params)
        p = probs.numpy().reshape(rows, n)
        out = _u32(pick).reshape(rows, split)
        KA = kept_all.numpy()
        units = world * split
        for r in range(rows):
            T, rnd = P[r, 0], P[r, 3]
            out[r] = NONE
            if T <= 0:
                continue
            vals = [float(KA[_gidx(u, r, rows, split)]) for u in range(units)]
            target = float(rnd) * max(sum(vals), 1e-20)
            thr = state["thr"][r]
            for c, (b, e) in enumerate(self._spans(n, split)):
                seg = p[r, b:e]
                run = sum(vals[: rank * split + c]) + np.cumsum(np.where(seg >= thr, seg, 0.0))
                hit = np.nonzero((run >= target) & (seg >= thr))[0]
                if hit.size:
                    out[r, c] = row_begin + b + int(hit[0])

    def finish(self, rows, split, world, params, cand_all, pick_all, state, out):
        P = _params(params)
        C = _u32(cand_all).reshape(-1, 4)
        PA = _u32(pick_all)
        o = _u32(out)
        units = world * split
        for r in range(rows):
            if P[r, 0] <= 0:
                bv, bi = f32(-1e30), NONE
                for u in range(units):
                    c = C[_gidx(u, r, rows, split)]
                    v = c[0:1].view(f32)[0]
                    if v > bv or (v == bv and c[1] < bi):
                        bv, bi = v, int(c[1])
                o[r] = 0 if bi == NONE else bi
            else:
                best = min(int(PA[_gidx(u, r, rows, split)]) for u in range(units))
                o[r] = state["garg"][r] if best == NONE else best
