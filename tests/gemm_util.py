"""ctypes view of include/pufferlean_b200_testing.h for the GEMM kernel tests."""
import ctypes as C

import pufferlean_b200 as plb

EPI_F32, EPI_BF16, EPI_FWD, EPI_DGRAD, EPI_PPO = 0, 1, 2, 3, 4


class GemmArgs(C.Structure):
    _fields_ = [
        ("a", C.c_void_p), ("a_rows", C.c_long), ("a_cols", C.c_long), ("a_ld", C.c_long), ("a_bstride", C.c_long),
        ("a_mn", C.c_int),
        ("b", C.c_void_p), ("b_rows", C.c_long), ("b_cols", C.c_long), ("b_ld", C.c_long), ("b_bstride", C.c_long),
        ("b_mn", C.c_int),
        ("M", C.c_int), ("N", C.c_int), ("K", C.c_int), ("bn", C.c_int), ("epi", C.c_int), ("batch", C.c_int),
        ("k_splits", C.c_int),
        ("out", C.c_void_p), ("ldo", C.c_long), ("out_bstride", C.c_long), ("out_rows", C.c_int),
        ("out_cols", C.c_int),
        ("alpha", C.c_float), ("beta", C.c_float),
        ("aux", C.c_void_p), ("ld_aux", C.c_long), ("aux_bstride", C.c_long),
        ("bias", C.c_void_p),
        ("out2", C.c_void_p), ("ldo2", C.c_long),
        ("colsum", C.c_void_p), ("ld_colsum", C.c_long),
        ("act", C.c_int),
        ("act_idx", C.c_void_p), ("adv", C.c_void_p), ("ret", C.c_void_p), ("olp", C.c_void_p), ("ov", C.c_void_p),
        ("A", C.c_int), ("vf", C.c_float), ("ent", C.c_float), ("clip", C.c_float), ("vfclip", C.c_float),
        ("newlp", C.c_void_p), ("newval", C.c_void_p), ("loss_part", C.c_void_p),
    ]


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def run(args: GemmArgs):
    L = plb.lib()
    L.pl_test_gemm.argtypes = [C.POINTER(GemmArgs), C.c_void_p]
    rc = L.pl_test_gemm(C.byref(args), None)
    if rc != 0:
        raise plb.PufferError(L.pl_last_error().decode())


def device_error():
    L = plb.lib()
    v = C.c_uint(0)
    L.pl_test_device_error(C.byref(v))
    return v.value


def operand(t, mn=False):
    """(ptr, rows, cols, ld) of a 2-D bf16 torch tensor (contiguous rows)."""
    assert t.dim() == 2 and t.stride(1) == 1
    return C.c_void_p(t.data_ptr()), t.shape[0], t.shape[1], t.stride(0)


def gemm(opA, opB, M, N, K, a_mn=False, b_mn=False, bn=128, epi=EPI_F32, out=None, ldo=None, out_rows=None,
         out_cols=None, **kw):
    g = GemmArgs()
    g.a, g.a_rows, g.a_cols, g.a_ld = operand(opA)
    g.b, g.b_rows, g.b_cols, g.b_ld = operand(opB)
    g.a_mn, g.b_mn = int(a_mn), int(b_mn)
    g.M, g.N, g.K, g.bn, g.epi, g.batch, g.k_splits = M, N, K, bn, epi, 1, kw.pop("k_splits", 1)
    g.out = ptr(out)
    g.ldo = ldo if ldo is not None else out.stride(0)
    g.out_rows = out_rows if out_rows is not None else M
    g.out_cols = out_cols if out_cols is not None else N
    g.alpha, g.beta = kw.pop("alpha", 1.0), kw.pop("beta", 0.0)
    for k, v in kw.items():
        if hasattr(v, "data_ptr"):
            setattr(g, k, ptr(v))
        else:
            setattr(g, k, v)
    run(g)
    return g
