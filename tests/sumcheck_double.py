"""A numpy stand-in for the GPU stepwise sumcheck session (CPU tests only).

It implements the same five calls as zkml_b200.distributed.GpuSumcheckSession
(load_m31 / load_qm31 / round / export / finalize) with plain numpy QM31
arithmetic, so the multi-rank orchestration can be tested with gloo ranks on a
machine without a GPU.  It is test infrastructure, never a product path.
"""
import numpy as np

P = (1 << 31) - 1


def qmul(x, y):
    """Element-wise QM31 product of (..., 4) int64 arrays: (a + b i) + (c + d i) u, u^2 = 2 + i."""
    a, b, c, d = (x[..., k] for k in range(4))
    e, f, g, h = (y[..., k] for k in range(4))
    # X*Z with X = a + b i, Z = e + f i
    xz_r = (a * e - b * f) % P
    xz_i = (a * f + b * e) % P
    yw_r = (c * g - d * h) % P
    yw_i = (c * h + d * g) % P
    # (2 + i) * YW
    t_r = (2 * yw_r - yw_i) % P
    t_i = (yw_r + 2 * yw_i) % P
    r_r = ((a * g - b * h) % P + (c * e - d * f) % P) % P
    r_i = ((a * h + b * g) % P + (c * f + d * e) % P) % P
    return np.stack([(xz_r + t_r) % P, (xz_i + t_i) % P, r_r, r_i], axis=-1)


class NumpySumcheckSession:
    def load_m31(self, a, b):
        a = np.asarray(a, np.int64) % P
        b = np.asarray(b, np.int64) % P
        self.a = np.zeros((len(a), 4), np.int64)
        self.b = np.zeros((len(b), 4), np.int64)
        self.a[:, 0] = a
        self.b[:, 0] = b

    def load_qm31(self, a, b):
        self.a = np.asarray(a, np.int64).reshape(-1, 4).copy()
        self.b = np.asarray(b, np.int64).reshape(-1, 4).copy()

    def length(self):
        return len(self.a)

    def _sums(self):
        h = len(self.a) // 2
        alo, ahi, blo, bhi = self.a[:h], self.a[h:], self.b[:h], self.b[h:]
        s0 = qmul(alo, blo).sum(0) % P
        s1 = qmul(ahi, bhi).sum(0) % P
        s2 = qmul((2 * ahi - alo) % P, (2 * bhi - blo) % P).sum(0) % P
        return np.concatenate([s0, s1, s2]).astype(np.uint32)

    def _fold(self, alpha):
        al = np.broadcast_to(np.asarray(alpha, np.int64), (len(self.a) // 2, 4))
        h = len(self.a) // 2
        self.a = (self.a[:h] + qmul(al, (self.a[h:] - self.a[:h]) % P)) % P
        self.b = (self.b[:h] + qmul(al, (self.b[h:] - self.b[:h]) % P)) % P

    def round(self, alpha=None):
        if alpha is not None:
            self._fold(alpha)
        return self._sums()

    def export(self):
        return self.a.astype(np.uint32), self.b.astype(np.uint32)

    def finalize(self, alpha):
        self._fold(alpha)
        return self.a[0].astype(np.uint32), self.b[0].astype(np.uint32)
