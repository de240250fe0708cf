"""The minibatch row gather of the update (the device twin of lean_ffi_gather_minibatch,
ffi/pufferffi.c:1046-1081, and of the reference's device gathers k_gather_f32 / k_gather_f64,
ffi/puffercuda.cu:870-875) is bit-exact: every gathered row and scalar equals the reference's own
output, after the one conversion each column gets on upload (observations to f32 in the tight tier or
to bf16 in the bf16 tier, the scalars to f32 and the actions to int32).

The gather is run through pl_test_update_gather, which takes the same row range, the same shuffle
(translated into first-epoch positions when the observations were uploaded in that order) and the same
kernel as pl_update_run. Covered: the reference's golden output over three epochs with a ragged last
minibatch, rows that are and are not a multiple of the 16-byte vector, the padded bf16 rows, and the
first-epoch-order upload of the reference-shaped call (epoch 0 reads its rows in place, later epochs
through the translated shuffle)."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
vp = C.c_void_p


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _lib():
    L = plb.lib()
    from tests.test_gpu_dp import Desc
    L.pl_update_create.argtypes = [C.c_size_t, C.POINTER(Desc), C.POINTER(vp)]
    L.pl_update_set_columns.argtypes = [vp] * 9
    L.pl_update_run_columns.argtypes = [vp] * 8 + [C.c_double, vp]
    L.pl_update_destroy.argtypes = [vp]
    sz = C.c_size_t
    L.pl_test_update_gather.argtypes = [vp, sz, sz, vp, C.POINTER(sz), vp, vp, vp, vp, vp, C.POINTER(sz), vp]
    return L


class _Session:
    def __init__(self, NT, D, H, A, E, MB, bf16):
        from tests.test_gpu_dp import Arch, Desc
        self.L = _lib()
        self.P = O.param_count(D, H, A, 1)
        g = np.random.default_rng(NT + D)
        pm = np.zeros(2 * self.P)
        pm[:self.P] = g.uniform(-0.1, 0.1, self.P)
        self.h = plb.policy_load(pm, self.P)
        d = Desc(NT=NT, D=D, H=H, A=A, epochs=E, numMB=MB, arch=Arch(1, 0, None, 0), wd=0.0, mu=0.95, eps=1e-7,
                 vfCoef=0.5, entCoef=0.01, clipEps=0.2, vfClip=0.2, maxGradNorm=0.5, bf16=bf16, use_old_values=1,
                 rank=0, world=1, comm=None)
        self.u = vp()
        assert self.L.pl_update_create(self.h, C.byref(d), C.byref(self.u)) == 0, self.L.pl_last_error()
        self.NT, self.D, self.bf16 = NT, D, bf16

    def close(self):
        self.L.pl_update_destroy(self.u)
        plb.policy_free(self.h)

    def gather(self, e, m):
        n_max = self.NT
        re_max = max(64, -(-self.D // 64) * 64)
        rows = np.zeros(n_max * re_max, dtype=np.uint16 if self.bf16 else np.float32)
        act = np.zeros(n_max, dtype=np.int32)
        adv, ret, olp, ov = (np.zeros(n_max, dtype=np.float32) for _ in range(4))
        re, nmb = C.c_size_t(), C.c_size_t()
        rc = self.L.pl_test_update_gather(self.u, e, m, rows.ctypes.data, C.byref(re), act.ctypes.data,
                                          adv.ctypes.data, ret.ctypes.data, olp.ctypes.data, ov.ctypes.data,
                                          C.byref(nmb), None)
        assert rc == 0, self.L.pl_last_error()
        n, w = nmb.value, re.value
        return rows[:n * w].reshape(n, w), act[:n], adv[:n], ret[:n], olp[:n], ov[:n]


def _cols(NT, D, seed):
    g = np.random.default_rng(seed)
    return (g.standard_normal(NT * D) * 2.0, g.integers(0, 5, NT).astype(float), g.standard_normal(NT),
            g.standard_normal(NT), g.uniform(-4.0, -0.1, NT), g.standard_normal(NT))


def _bf16_bits(x64):
    """The session's conversion of f64 observations to bf16: to f32 to nearest, then to bf16 to nearest
    even (torch on the host performs the same two roundings)."""
    t = torch.from_numpy(np.ascontiguousarray(x64)).to(torch.float32).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


def _check_rows(sess, got, want_obs, D):
    rows = got[0]
    if sess.bf16:
        assert np.array_equal(rows[:, :D], _bf16_bits(want_obs).reshape(-1, D))
        assert not rows[:, D:].any()  # zero padding
    else:
        assert np.array_equal(rows, want_obs.astype(np.float32).reshape(-1, D))


def _minibatches(NT, E, MB):
    mb = NT // MB
    for e in range(E):
        for m in range(MB):
            lo, hi = m * mb, (NT if m + 1 == MB else (m + 1) * mb)
            yield e, m, lo, hi


def test_device_gather_equals_reference_golden_tight_tier():
    """The reference's lean_ffi_gather_minibatch outputs (tests/golden/gather_minibatch.npz, made by its
    compiled C) for every minibatch of three epochs, D = 9 (no 16-byte vectors), ragged last minibatch."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "gather_minibatch.npz"))
    NT, D, E, MB = (int(x) for x in g["meta"])
    s = _Session(NT, D, 16, 7, E, MB, 0)
    try:
        cols = [np.ascontiguousarray(x) for x in (g["obs"], g["acts"], g["advs"], g["rets"], g["olps"], g["rets"],
                                                  g["perm"])]
        assert s.L.pl_update_set_columns(s.u, *[x.ctypes.data for x in cols], None) == 0, s.L.pl_last_error()
        k = 0
        for e, m, lo, hi in _minibatches(NT, E, MB):
            n = hi - lo
            got = s.gather(e, m)
            assert got[1].size == n
            _check_rows(s, got, g["mbObs"][k * D:(k + n) * D], D)
            assert np.array_equal(got[1], g["mbAct"][k:k + n].astype(np.int32))
            for x, name in zip(got[2:5], ("mbAdv", "mbRet", "mbOlp")):
                assert np.array_equal(x, g[name][k:k + n].astype(np.float32)), name
            k += n
        assert k == E * NT
    finally:
        s.close()


@pytest.mark.parametrize("NT,D,E,MB,bf16", [(4099, 16, 3, 5, 0), (4133, 40, 2, 3, 1), (2053, 128, 2, 2, 1)])
def test_device_gather_equals_host_twin(NT, D, E, MB, bf16):
    """Against pl_gather_minibatch (bit-exact to the reference's golden output on the CPU): f32 rows in
    16-byte vectors, bf16 rows padded to 64 values, and rows wider than one vector pass per lane."""
    obs, acts, adv, ret, olp, ov = _cols(NT, D, NT)
    perm = O.shuffle_perm(NT, E, 0x5EED + NT)
    s = _Session(NT, D, 64, 5, E, MB, bf16)
    try:
        cols = [np.ascontiguousarray(x) for x in (obs, acts, adv, ret, olp, ov, perm)]
        assert s.L.pl_update_set_columns(s.u, *[x.ctypes.data for x in cols], None) == 0, s.L.pl_last_error()
        for e, m, lo, hi in _minibatches(NT, E, MB):
            idx = perm[e * NT + lo:e * NT + hi]
            want = plb.gather_minibatch(obs, acts, adv, ret, olp, idx, hi - lo, D)
            got = s.gather(e, m)
            _check_rows(s, got, want[0], D)
            assert np.array_equal(got[1], want[1].astype(np.int32))
            for x, w in zip(got[2:5], want[2:5]):
                assert np.array_equal(x, w.astype(np.float32))
            assert np.array_equal(got[5], ov[idx.astype(np.int64)].astype(np.float32))
    finally:
        s.close()


def test_device_gather_after_first_epoch_order_upload():
    """The reference-shaped call uploads observations in the first epoch's shuffle order while it runs:
    epoch 0 then reads its rows in place and later epochs read row pos[perm_e[k]] through the translated
    shuffle. Every epoch's rows must still be the reference's gathered rows."""
    NT, D, E, MB = 16384 + 5, 64, 3, 4
    obs, acts, adv, ret, olp, ov = _cols(NT, D, 9)
    perm = O.shuffle_perm(NT, E, 0xF1)
    s = _Session(NT, D, 64, 5, E, MB, 1)
    try:
        cols = [np.ascontiguousarray(x) for x in (obs, acts, adv, ret, olp, ov, perm)]
        assert s.L.pl_update_run_columns(s.u, *[x.ctypes.data for x in cols], 0.02, None) == 0, s.L.pl_last_error()
        for e, m, lo, hi in _minibatches(NT, E, MB):
            idx = perm[e * NT + lo:e * NT + hi]
            want = plb.gather_minibatch(obs, acts, adv, ret, olp, idx, hi - lo, D)
            got = s.gather(e, m)
            _check_rows(s, got, want[0], D)
            assert np.array_equal(got[1], want[1].astype(np.int32))
            assert np.array_equal(got[2], want[2].astype(np.float32))
    finally:
        s.close()
