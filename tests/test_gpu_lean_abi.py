"""The reference's Lean symbols through libpufferlean_lean.so on the GPU, with Lean FloatArray
objects built the way the Lean runtime lays them out (include/lean_compat)."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402
from oracle.oracle import FA  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
VP = C.c_void_p


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    plb.lib()
    return C.CDLL(os.path.join(os.path.dirname(plb.LIB_PATH), "libpufferlean_lean.so"))


def test_lean_cuda_vtrace_kat(lib):
    f = np.load(os.path.join(GOLD, "vtrace.npz"))
    B, T, g, l, rho, c = f["meta"]
    out = O.ref_call(lib, "lean_cuda_vtrace", VP, FA(f["rew"]), FA(f["val"]), FA(f["term"]), FA(f["imp"]), int(B),
                     int(T), g, l, rho, c)
    assert np.array_equal(O.read_float_array(out), f["adv"])


def test_lean_cuda_train_update_kat(lib):
    f = np.load(os.path.join(GOLD, "train_update.npz"))
    NT, D, H, A, E, MB, vf, ent, clip, lr, wd, mu, eps, seed = f["meta"]
    NT, D, H, A, E, MB = (int(x) for x in (NT, D, H, A, E, MB))
    perm = O.read_float_array(O.ref_call(lib, "lean_ffi_shuffle_perm", VP, NT, E, ("u64", int(seed))))
    out = O.ref_call(lib, "lean_cuda_train_update", VP, FA(f["pm0"]), FA(f["obs"]), FA(f["acts"]), FA(f["adv"]),
                     FA(f["rets"]), FA(f["olps"]), FA(perm), NT, D, H, A, E, MB, lr, wd, mu, eps, vf, ent, clip,
                     ("u8", 0))
    assert np.abs(O.read_float_array(out) - f["out"]).max() < 1e-3


def test_lean_resident_policy_round_trip(lib):
    f = np.load(os.path.join(GOLD, "train_update.npz"))
    NT, D, H, A, E, MB, vf, ent, clip, lr, wd, mu, eps, seed = f["meta"]
    NT, D, H, A, E, MB = (int(x) for x in (NT, D, H, A, E, MB))
    P = f["pm0"].size // 2
    r = O.ref_call(lib, "lean_cuda_policy_load", VP, FA(f["pm0"]), P, ("obj", 1))
    assert O.ctor_tag(r) == 0
    hobj = O.ctor_field(r, 0)
    # USize boxed as a scalar constructor: the handle is its 8-byte payload
    handle = int.from_bytes(C.string_at(hobj + 8, 8), "little")
    perm = O.read_float_array(O.ref_call(lib, "lean_ffi_shuffle_perm", VP, NT, E, ("u64", int(seed))))
    r = O.ref_call(lib, "lean_cuda_train_update_resident", VP, handle, FA(f["obs"]), FA(f["acts"]), FA(f["adv"]),
                   FA(f["rets"]), FA(f["olps"]), FA(np.zeros(0)), FA(perm), NT, D, H, A, E, MB, lr, wd, mu, eps, vf,
                   ent, clip, 0.0, 0.0, ("u8", 0), ("obj", 1))
    assert O.ctor_tag(r) == 0
    p0 = O.read_float_array(O.ctor_field(r, 0))
    r = O.ref_call(lib, "lean_cuda_policy_download", VP, handle, P, ("obj", 1))
    pm = O.read_float_array(O.ctor_field(r, 0))
    assert p0[0] == pm[0]
    assert np.abs(pm - f["out"]).max() < 1e-3
    r = O.ref_call(lib, "lean_cuda_policy_free", VP, handle, ("obj", 1))
    assert O.ctor_tag(r) == 0
