"""The host-side bf16 rounding of observation rows (f64 -> f32 to nearest, then f32 -> bf16 to nearest
even, NaN -> 0x7FFF, rows zero-padded to Dp) against a numpy restatement, on CPU: ties both ways,
subnormals, signed zeros, overflow to infinity, NaN."""
import ctypes as C

import numpy as np

import pufferlean_b200 as plb


def _ref(x, D, Dp):
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r[nan] = 0x7FFF
    out = np.zeros((x.size // D, Dp), dtype=np.uint16)
    out[:, :D] = r.reshape(-1, D)
    return out.ravel()


def test_host_rounding_matches_restatement():
    rng = np.random.default_rng(3)
    D, Dp, rows = 24, 32, 4096
    x = rng.standard_normal(rows * D) * np.exp(rng.uniform(-100, 100, rows * D))
    ties = (np.arange(512) + 256.0) * 2.0 ** -8 + 2.0 ** -17
    x[:512] = ties
    x[512:1024] = -ties
    x[1024:1040] = [0.0, -0.0, 1e-40, -1e-45, 3.4e38, 3.5e38, -1e39, np.inf, -np.inf, np.nan, 2.0 ** -149,
                    2.0 ** -150, 65504.0, 1.0 + 2 ** -9, 1.0 + 3 * 2 ** -9, -(1.0 + 2 ** -9)]
    L = plb.lib()
    L.pl_test_round_rows_bf16.argtypes = [C.POINTER(C.c_double), C.c_long, C.c_int, C.c_int,
                                          C.POINTER(C.c_uint16)]
    out = np.full(rows * Dp, 0xABCD, dtype=np.uint16)
    with np.errstate(over="ignore"):
        want = _ref(x, D, Dp)
    assert L.pl_test_round_rows_bf16(x.ctypes.data_as(C.POINTER(C.c_double)), rows, D, Dp,
                                     out.ctypes.data_as(C.POINTER(C.c_uint16))) == 0
    assert np.array_equal(out, want)
