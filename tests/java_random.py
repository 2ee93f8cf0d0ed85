"""java.util.Random (the published 48-bit LCG of its Javadoc), vectorised,
to rebuild the reference tests' Random(42) fixtures bit for bit."""
import numpy as np

_A = 0x5DEECE66D
_C = 0xB
_MASK = (1 << 48) - 1
_BLOCK = 1 << 16


def _mulmod48(a: int, s: np.ndarray) -> np.ndarray:
    a_lo, a_hi = np.uint64(a & 0xFFFFFF), np.uint64(a >> 24)
    s_lo, s_hi = s & np.uint64(0xFFFFFF), s >> np.uint64(24)
    mid = (a_hi * s_lo + a_lo * s_hi) & np.uint64(0xFFFFFF)
    return (a_lo * s_lo + (mid << np.uint64(24))) & np.uint64(_MASK)


class JavaRandom:
    def __init__(self, seed: int):
        s = (seed ^ _A) & _MASK
        first = np.empty(_BLOCK, np.uint64)
        for i in range(_BLOCK):
            s = (s * _A + _C) & _MASK
            first[i] = s
        self._block = first
        # Jump of one block: s -> A_B * s + C_B (mod 2^48).
        a_b, c_b = 1, 0
        for _ in range(_BLOCK):
            a_b, c_b = (a_b * _A) & _MASK, (c_b * _A + _C) & _MASK
        self._ab, self._cb = a_b, c_b
        self._pos = 0

    def _next_seeds(self, n: int) -> np.ndarray:
        out = np.empty(n, np.uint64)
        k = 0
        while k < n:
            if self._pos == _BLOCK:
                self._block = (_mulmod48(self._ab, self._block) + np.uint64(self._cb)) & np.uint64(_MASK)
                self._pos = 0
            take = min(n - k, _BLOCK - self._pos)
            out[k:k + take] = self._block[self._pos:self._pos + take]
            self._pos += take
            k += take
        return out

    def next_floats(self, n: int) -> np.ndarray:
        """n successive nextFloat() values: next(24) / 2^24."""
        return ((self._next_seeds(n) >> np.uint64(24)).astype(np.float64) / float(1 << 24)).astype(np.float32)


def random_array(rng: JavaRandom, size: int, scale: float) -> np.ndarray:
    """TransformerBlockTest.randomArray: (nextFloat() - 0.5f) * 2 * scale in float."""
    f = rng.next_floats(size)
    return ((f - np.float32(0.5)) * np.float32(2)) * np.float32(scale)
