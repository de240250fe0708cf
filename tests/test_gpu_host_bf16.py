"""Host observations in the bf16 tier are rounded to bf16 on the host threads (f64 -> f32 to nearest,
f32 -> bf16 to nearest even) and copied as bf16, a quarter of the f64 bytes: the device copy and the
whole update are bit-identical to copying the f64 rows and converting them on the device, including
rounding ties, subnormals, signed zeros, infinities after the f32 step and values beyond the bf16
range, for row widths with and without padding, from pageable and from pinned memory. Rows of 64 or
more values are uploaded by the reference-shaped call in the first epoch's shuffle order, one
minibatch's rows ahead of its kernels, and later epochs read them through the translated shuffle;
narrower pinned rows are split between the host rounding and f64 copies converted on the device."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _mode(m):
    L = plb.lib()
    L.pl_test_host_bf16.argtypes = [C.c_int]
    return L.pl_test_host_bf16(m)


def _edge_values(n, rng):
    f32 = np.float32
    ties = (np.arange(n) % 512 + 256).astype(np.float64) * 2.0 ** -8 + 2.0 ** -17  # halfway between bf16s
    ties = ties * np.where(rng.random(n) < 0.5, -1.0, 1.0)
    special = np.array([0.0, -0.0, 1e-40, -1e-40, 3.4e38, -3.4e38, 1e39, -1e39, 6.1e-5, 65504.0, 1.0 + 2 ** -30,
                        float(f32(1.0) + f32(2 ** -8)), 2.0 ** -126, 2.0 ** -149])
    out = rng.standard_normal(n) * np.exp(rng.uniform(-20, 20, n))
    out[: n // 4] = ties[: n // 4]
    out[n // 4: n // 4 + special.size] = special
    return out


@pytest.mark.parametrize("D,pinned,MB", [(64, False, 4), (20, False, 4), (64, True, 4), (72, True, 3),
                                         (20, True, 4), (128, False, 1)])
def test_host_rounding_bit_identical(D, pinned, MB):
    """Against f64 copies converted on the device in column order: rows of >= 64 values go in the first
    epoch's order, minibatch by minibatch (3 minibatches: a ragged last one); narrower pinned rows are
    split between the host rounding and device conversion."""
    from tests.test_gpu_update import _problem, _run_resident
    NT, H, A, L, E = (65536 if D < 64 else 16384), 128, 5, 1, 2
    P, pm, obs, acts, adv, ret, olp, ov = _problem(NT, D, H, A, L, 61 + D, 1)
    rng = np.random.default_rng(D)
    obs = obs.copy()
    # rounding ties, subnormals and signed zeros among ordinary values (the extremes, which would
    # overflow the network, are covered elementwise below)
    x = _edge_values(NT * D // 8, rng)
    obs[: NT * D // 8] = np.where(np.abs(x) < 8.0, x, np.sign(x) * 2.0 ** -130)
    perm = O.shuffle_perm(NT, E, 82)
    keep = None
    if pinned:
        keep = torch.from_numpy(obs).pin_memory()
        obs = keep.numpy()
    args = (acts, adv, ret, olp, ov, perm, NT, D, H, A, E, MB, 0.02, 0.2, 0.5, 1)
    prev = _mode(1)
    try:
        host, _ = _run_resident(pm, P, (L, 1), obs, *args)
        _mode(0)
        dev, _ = _run_resident(pm, P, (L, 1), obs, *args)
    finally:
        _mode(prev)
    assert np.isfinite(host).all()
    assert np.array_equal(host, dev)
    assert not np.array_equal(host[:P], pm[:P])


def test_invalid_shuffle_entry_is_an_error():
    """A first-epoch shuffle entry outside [0, NT) (or not an integer) fails the call with an error
    instead of reading outside the host rows."""
    from tests.test_gpu_update import _problem, _run_resident
    NT, D, H, A, L, E, MB = 16384, 64, 128, 5, 1, 2, 4
    P, pm, obs, acts, adv, ret, olp, ov = _problem(NT, D, H, A, L, 5, 1)
    for bad in (float(NT), -1.0, 2.5):
        perm = O.shuffle_perm(NT, E, 3).copy()
        perm[NT // 2 + 7] = bad
        with pytest.raises(AssertionError, match="shuffle entry"):
            _run_resident(pm, P, (L, 1), obs, acts, adv, ret, olp, ov, perm, NT, D, H, A, E, MB, 0.02, 0.2, 0.5, 1)


def test_host_rounding_matches_device_conversion_elementwise():
    """The conversion itself over special values (no network in between): torch's f32 -> bf16 on the
    GPU is the reference for the rounding of the f32 values."""
    rng = np.random.default_rng(5)
    x = _edge_values(1 << 16, rng)
    want = torch.from_numpy(x).to(torch.float32).cuda().to(torch.bfloat16).view(torch.int16).cpu().numpy()
    L = plb.lib()
    L.pl_test_round_rows_bf16.argtypes = [C.POINTER(C.c_double), C.c_long, C.c_int, C.c_int,
                                          C.POINTER(C.c_uint16)]
    out = np.zeros(x.size, dtype=np.uint16)
    assert L.pl_test_round_rows_bf16(x.ctypes.data_as(C.POINTER(C.c_double)), x.size // 64, 64, 64,
                                     out.ctypes.data_as(C.POINTER(C.c_uint16))) == 0
    assert np.array_equal(out.view(np.int16), want)


def test_session_run_columns_equals_set_columns_and_run():
    """pl_update_run_columns (rows uploaded in the first epoch's order during the run) against
    pl_update_set_columns + pl_update_run on a session: bit-identical parameters, twice in a row on the
    same session (the second call's upload waits for nothing stale)."""
    from tests.test_gpu_dp import Arch, Desc
    from tests.test_gpu_update import _problem
    NT, D, H, A, L, E, MB = 16384, 96, 128, 5, 2, 2, 3
    P, pm, obs, acts, adv, ret, olp, ov = _problem(NT, D, H, A, L, 77, 1)
    L_ = plb.lib()
    vp = C.c_void_p
    L_.pl_update_create.argtypes = [C.c_size_t, C.POINTER(Desc), C.POINTER(vp)]
    L_.pl_update_set_columns.argtypes = [vp] * 9
    L_.pl_update_run.argtypes = [vp, C.c_double, vp]
    L_.pl_update_run_columns.argtypes = [vp] * 8 + [C.c_double, vp]
    L_.pl_update_destroy.argtypes = [vp]
    outs = []
    for combined in (False, True):
        h = plb.policy_load(pm, P)
        d = Desc(NT=NT, D=D, H=H, A=A, epochs=E, numMB=MB, arch=Arch(L, 1, None, 0), wd=0.0, mu=0.95, eps=1e-7,
                 vfCoef=0.5, entCoef=0.01, clipEps=0.2, vfClip=0.2, maxGradNorm=0.5, bf16=1, use_old_values=1,
                 rank=0, world=1, comm=None)
        u = vp()
        assert L_.pl_update_create(h, C.byref(d), C.byref(u)) == 0, L_.pl_last_error()
        try:
            for i in range(2):
                perm = np.ascontiguousarray(O.shuffle_perm(NT, E, 90 + i), dtype=np.float64)
                cols = [np.ascontiguousarray(x, dtype=np.float64) for x in (obs, acts, adv, ret, olp, ov)]
                ptrs = [x.ctypes.data for x in cols] + [perm.ctypes.data]
                if combined:
                    rc = L_.pl_update_run_columns(u, *ptrs, 0.02, None)
                else:
                    rc = L_.pl_update_set_columns(u, *ptrs, None)
                    rc = rc or L_.pl_update_run(u, 0.02, None)
                assert rc == 0, L_.pl_last_error()
            torch.cuda.synchronize()
        finally:
            L_.pl_update_destroy(u)
        outs.append(plb.policy_download(h, P))
        plb.policy_free(h)
    assert np.isfinite(outs[0]).all()
    assert np.array_equal(outs[0], outs[1])
    assert not np.array_equal(outs[0][:P], pm[:P])
