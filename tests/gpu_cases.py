"""Shared inputs for the GPU parity tests: seeded tiles and fault patterns."""
import numpy as np


def tiles(orc, M, K, N, seed_a=123456, seed_b=987654, dist="uniform"):
    A = orc.fill_random(M * K, seed_a, dist).reshape(M, K)
    B = orc.fill_random(K * N, seed_b, dist).reshape(K, N)
    return A, B


def product_f64(A, B):
    """A reference product rounded to float32 (stands in for an SGEMM output)."""
    return (A.astype(np.float64) @ B.astype(np.float64)).astype(np.float32)


def add_fault(C, r, c, delta):
    C = C.copy()
    C[r, c] = np.float32(C[r, c] + np.float32(delta))
    return C


def flip(C, r, c, bit):
    C = C.copy()
    u = C.view(np.uint32)
    u[r, c] ^= np.uint32(1 << bit)
    return C
