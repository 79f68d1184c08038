"""Seeded synthetic inputs for the parity tests, restating the reference harnesses' generators.

- hashu / normal: bench/emugemm_test.cpp:19-25 (hash-based Box-Muller; seeds 12345 for A, 67890 for B)
- uniform: U[-1,1] from the same hash
- family2: the adversarial cancellation family of bench/emu_adversarial.cpp:32-40 / bench/rho_sweep.cpp:72-82,
  A = [G|G], B = [H; -H + d*G2], d = 0.6366*sqrt(2K)/rho
- oscillatory: A[i,k] = exp(-((k/K - i/M)^2)/0.01), B[k,j] = cos(2*pi*f_j*k/K + phi_j) with the frequencies
  set per case so that the cancellation ratio spans about 1.2 to 3000
- wide_range: N(0,1) * 2^e with e uniform in [-20, 20] per element (full FP32 exponent-range stress)
All values are computed in float32 with numpy; the FP64 ground truth is always taken from the same arrays.
"""
from __future__ import annotations

import numpy as np

_M32 = np.uint64(0xFFFFFFFF)


def hashu(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.uint64) & _M32
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & _M32
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & _M32
    x ^= x >> np.uint64(16)
    return x


def _unif(idx: np.ndarray, seed: int) -> np.ndarray:
    h = hashu((idx.astype(np.uint64) & _M32) ^ np.uint64(seed))
    return (h >> np.uint64(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)


def _gauss(idx: np.ndarray, seed: int) -> np.ndarray:
    u1 = np.maximum(_unif(idx, seed), np.float32(1e-7))
    u2 = _unif(idx, seed + 0x9E37)
    return (np.sqrt(np.float32(-2.0) * np.log(u1)) * np.cos(np.float32(6.2831853) * u2)).astype(np.float32)


def normal(shape, seed: int, scale: float = 1.0) -> np.ndarray:
    """bench/emugemm_test.cpp:21-25."""
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.uint64)
    a = hashu((i & _M32) ^ np.uint64(seed))
    b = hashu(((i >> np.uint64(32)) ^ ((a + np.uint64(0x9E3779B9)) & _M32)) & _M32)
    u1 = np.maximum((a >> np.uint64(8)).astype(np.float32) * np.float32(1.0 / 16777216.0), np.float32(1e-7))
    u2 = (b >> np.uint64(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    x = np.float32(scale) * np.sqrt(np.float32(-2.0) * np.log(u1)) * np.cos(np.float32(6.2831853) * u2)
    return x.astype(np.float32).reshape(shape)


def uniform(shape, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    u = _unif(np.arange(n, dtype=np.uint64), seed)
    return (np.float32(2.0) * u - np.float32(1.0)).astype(np.float32).reshape(shape)


def wide_range(shape, seed: int, emax: int = 20) -> np.ndarray:
    n = int(np.prod(shape))
    x = normal((n,), seed)
    e = (hashu(np.arange(n, dtype=np.uint64) ^ np.uint64(seed + 0x51ED)) % np.uint64(2 * emax + 1)).astype(np.int32)
    return np.ldexp(x, e - emax).astype(np.float32).reshape(shape)


def family2(M: int, N: int, K: int, rho: float) -> tuple[np.ndarray, np.ndarray]:
    """bench/emu_adversarial.cpp:32-40 (A seed 31337, B seeds 71993 / 55555)."""
    half = K // 2
    r = np.arange(M, dtype=np.uint64)[:, None]
    c = np.arange(K, dtype=np.uint64)[None, :]
    A = _gauss(r * np.uint64(half) + (c % np.uint64(half)), 31337)
    d = np.float32(0.6366 * np.sqrt(2.0 * K) / rho)
    k = np.arange(K, dtype=np.uint64)[:, None]
    j = np.arange(N, dtype=np.uint64)[None, :]
    base = _gauss((k % np.uint64(half)) * np.uint64(N) + j, 71993)
    lin = k * np.uint64(N) + j
    B = np.where(k < np.uint64(half), base, -base + d * _gauss(lin, 55555)).astype(np.float32)
    return np.ascontiguousarray(A, np.float32), np.ascontiguousarray(B, np.float32)


def oscillatory(M: int, N: int, K: int, f0: float, seed: int = 977) -> tuple[np.ndarray, np.ndarray]:
    """A[i,k] = exp(-((k/K - i/M)^2)/0.01): Gaussian bumps sliding along K; B[k,j] = cos(2 pi f_j k / K + phi_j)
    with f_j = f0 + u_j, u_j ~ U[0,1) per column and a random phase. The inner product of a bump with a fast
    oscillation nearly vanishes, so the cancellation ratio grows with f0 (measured in FP64 at 512x512x8192:
    f0 = 1.3 -> rho ~ 1.2, f0 = 11 -> ~30, f0 = 1150 -> ~3000; the bumps truncated at the ends of [0,1) make
    it grow linearly in f0)."""
    i = np.arange(M, dtype=np.float64)[:, None] / M
    k = np.arange(K, dtype=np.float64)[None, :] / K
    A = np.exp(-((k - i) ** 2) / 0.01).astype(np.float32)
    u = _unif(np.arange(N, dtype=np.uint64), seed).astype(np.float64)
    f = f0 + u
    ph = 2 * np.pi * _unif(np.arange(N, dtype=np.uint64), seed + 1).astype(np.float64)
    kk = np.arange(K, dtype=np.float64)[:, None]
    B = np.cos(2 * np.pi * f[None, :] * kk / K + ph[None, :]).astype(np.float32)
    return np.ascontiguousarray(A), np.ascontiguousarray(B)
