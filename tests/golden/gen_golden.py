"""Regenerate the golden fixtures in tests/golden/ from the reference's own compiled C.

Run in the build container (the reference tree must be present and no GPU visible):

    make -C oracle all ref && python tests/golden/gen_golden.py [--only gather]

Inputs are the seeded known-answer inputs of the reference's verify-* modes (oracle/kat.py).
Outputs come from the reference's C compiled from its sources by oracle/Makefile:
ffi/pufferffi.c and ffi/pufferblas.c (libref_cpu.so) and the host fallback loops of
ffi/puffercuda.cu (libref_cudafb.so; with no device those loops are what its entry points run).
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import kat  # noqa: E402
from oracle import oracle as O  # noqa: E402
from oracle.oracle import FA, ref_call  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
VP = __import__("ctypes").c_void_p


def arr(p):
    return O.read_float_array(p)


def unpack5(tup):
    """(a, (b, (c, (d, e)))) of the reference's Prod constructors -> five arrays."""
    out = []
    for _ in range(4):
        out.append(arr(O.ctor_field(tup, 0)))
        tup = O.ctor_field(tup, 1)
    out.append(arr(tup))
    return out


def gather_fixture(cpu):
    """lean_ffi_gather_minibatch over every minibatch of three shuffled epochs (ragged last minibatch,
    a row width that is not a multiple of the vector width), and lean_ffi_slice on a few ranges."""
    rng = kat.Rng(0x6A7E)
    NT, D, E, MB = 203, 9, 3, 4
    obs = np.array([rng.randF(-3.0, 3.0) for _ in range(NT * D)])
    acts = np.array([float(rng.next() % 7) for _ in range(NT)])
    advs = np.array([rng.randF(-2.0, 2.0) for _ in range(NT)])
    rets = np.array([rng.randF(-2.0, 2.0) for _ in range(NT)])
    olps = np.array([rng.randF(-4.0, -0.1) for _ in range(NT)])
    perm = arr(ref_call(cpu, "lean_ffi_shuffle_perm", VP, NT, E, ("u64", 0x6A7E)))
    mb = NT // MB
    outs = [[] for _ in range(5)]
    for e in range(E):
        for m in range(MB):
            lo, hi = m * mb, (NT if m + 1 == MB else (m + 1) * mb)
            idx = perm[e * NT + lo:e * NT + hi]
            got = unpack5(ref_call(cpu, "lean_ffi_gather_minibatch", VP, FA(obs), FA(acts), FA(advs), FA(rets),
                                   FA(olps), FA(idx), hi - lo, D))
            for i in range(5):
                outs[i].append(got[i])
    slices = [(0, 5), (17, 100), (NT * D - 3, 3), (40, 0)]
    sl = {f"slice{i}": arr(ref_call(cpu, "lean_ffi_slice", VP, FA(obs), off, ln)) for i, (off, ln) in enumerate(slices)}
    np.savez(os.path.join(OUT, "gather_minibatch.npz"), obs=obs, acts=acts, advs=advs, rets=rets, olps=olps, perm=perm,
             mbObs=np.concatenate(outs[0]), mbAct=np.concatenate(outs[1]), mbAdv=np.concatenate(outs[2]),
             mbRet=np.concatenate(outs[3]), mbOlp=np.concatenate(outs[4]), slices=np.array(slices),
             meta=np.array([NT, D, E, MB]), **sl)


def main():
    cpu = O.ref_cpu()
    if "--only" in sys.argv and sys.argv[sys.argv.index("--only") + 1] == "gather":
        gather_fixture(cpu)
        return
    cfb = O.ref_cudafb()
    out = {}
    gather_fixture(cpu)

    k = kat.kat_vtrace()
    a = arr(ref_call(cfb, "lean_cuda_vtrace", VP, FA(k["rew"]), FA(k["val"]), FA(k["term"]), FA(k["imp"]), k["B"],
                     k["T"], k["gamma"], k["lam"], k["rho"], k["c"]))
    np.savez(os.path.join(OUT, "vtrace.npz"), adv=a, **{x: k[x] for x in ("rew", "val", "term", "imp")},
             meta=np.array([k["B"], k["T"], k["gamma"], k["lam"], k["rho"], k["c"]]))

    k = kat.kat_vtrace_mingru()
    a = arr(ref_call(cfb, "lean_cuda_vtrace_mingru", VP, FA(k["rew"]), FA(k["val"]), FA(k["term"]), FA(k["imp"]),
                     FA(k["bootv"]), k["B"], k["T"], k["gamma"], k["lam"], k["rho"], k["c"]))
    np.savez(os.path.join(OUT, "vtrace_mingru.npz"), adv=a,
             **{x: k[x] for x in ("rew", "val", "term", "imp", "bootv")},
             meta=np.array([k["B"], k["T"], k["gamma"], k["lam"], k["rho"], k["c"]]))

    k = kat.kat_muon()
    d = {"meta": np.array([k["lr"], k["wd"], k["mu"], k["eps"]])}
    for i, cs in enumerate(k["cases"]):
        o = arr(ref_call(cfb, "lean_cuda_muon_stepmat", VP, FA(cs["W"]), FA(cs["G"]), FA(cs["M"]), cs["rows"],
                         cs["cols"], k["lr"], k["wd"], k["mu"], k["eps"]))
        d.update({f"W{i}": cs["W"], f"G{i}": cs["G"], f"M{i}": cs["M"], f"out{i}": o,
                  f"shape{i}": np.array([cs["rows"], cs["cols"]])})
    np.savez(os.path.join(OUT, "muon_stepmat.npz"), **d)

    k = kat.kat_advnorm()
    a = arr(ref_call(cfb, "lean_cuda_adv_normalize", VP, FA(k["adv"]), k["adv"].size))
    np.savez(os.path.join(OUT, "advnorm.npz"), adv=k["adv"], out=a)

    k = kat.kat_muon_cpu()
    o = arr(ref_call(cpu, "lean_ffi_muon_step_mlp", VP, FA(np.concatenate([k["params"], k["mom"]])), FA(k["grad"]),
                     k["H"], k["D"], k["O"], k["gscale"], k["lr"], k["wd"], k["mu"], k["eps"]))
    np.savez(os.path.join(OUT, "muon_cpu.npz"), params=k["params"], grad=k["grad"], mom=k["mom"], out=o,
             meta=np.array([k["H"], k["D"], k["O"], k["gscale"], k["lr"], k["wd"], k["mu"], k["eps"]]))

    k = kat.kat_ppo_grad()
    args = (FA(k["params"]), FA(k["obs"]), FA(k["acts"]), FA(k["advs"]), FA(k["rets"]), FA(k["olps"]))
    g_blas = arr(ref_call(cpu, "lean_ffi_mlp_ppo_grad_batch_blas", VP, *args, k["N"], k["H"], k["D"], k["A"],
                          k["vf"], k["ent"], k["clip"]))
    args = (FA(k["params"]), FA(k["obs"]), FA(k["acts"]), FA(k["advs"]), FA(k["rets"]), FA(k["olps"]))
    g_scal = arr(ref_call(cpu, "lean_ffi_mlp_ppo_grad_batch", VP, *args, k["N"], k["H"], k["D"], k["A"], k["vf"],
                          k["ent"], k["clip"]))
    ov = np.array([kat.Rng(0xC11F + i).randF(-1.0, 1.0) for i in range(k["N"])])
    args = (FA(k["params"]), FA(k["obs"]), FA(k["acts"]), FA(k["advs"]), FA(k["rets"]), FA(k["olps"]), FA(ov))
    g_vc = arr(ref_call(cpu, "lean_ffi_mlp_ppo_grad_batch_vclip", VP, *args, k["N"], k["H"], k["D"], k["A"], k["vf"],
                        k["ent"], k["clip"], 0.2))
    np.savez(os.path.join(OUT, "ppo_grad.npz"), g_blas=g_blas, g_scalar=g_scal, g_vclip=g_vc, ov=ov,
             **{x: k[x] for x in ("params", "obs", "acts", "advs", "rets", "olps")},
             meta=np.array([k["N"], k["D"], k["H"], k["A"], k["vf"], k["ent"], k["clip"], 0.2]))

    k = kat.kat_train_step()
    advN = arr(ref_call(cfb, "lean_cuda_adv_normalize", VP, FA(k["adv"]), k["N"]))
    g = arr(ref_call(cpu, "lean_ffi_mlp_ppo_grad_batch_blas", VP, FA(k["params"]), FA(k["obs"]), FA(k["acts"]),
                     FA(advN), FA(k["rets"]), FA(k["olps"]), k["N"], k["H"], k["D"], k["A"], k["vf"], k["ent"],
                     k["clip"]))
    pm = arr(ref_call(cpu, "lean_ffi_muon_step_mlp", VP, FA(np.concatenate([k["params"], k["mom"]])), FA(g), k["H"],
                      k["D"], k["A"] + 1, 1.0 / k["N"], k["lr"], k["wd"], k["mu"], k["eps"]))
    np.savez(os.path.join(OUT, "train_step.npz"), out=pm, advN=advN, grad=g,
             **{x: k[x] for x in ("params", "mom", "obs", "acts", "adv", "rets", "olps")},
             meta=np.array([k["N"], k["D"], k["H"], k["A"], k["vf"], k["ent"], k["clip"], k["lr"], k["wd"], k["mu"],
                            k["eps"]]))

    k = kat.kat_train_update()
    NT, D, H, A, E, MB = k["NT"], k["D"], k["H"], k["A"], k["epochs"], k["numMB"]
    perm = arr(ref_call(cpu, "lean_ffi_shuffle_perm", VP, NT, E, ("u64", k["perm_seed"])))
    pm = k["pm0"].copy()
    mb = NT // MB
    for e in range(E):
        for m in range(MB):
            lo, hi = m * mb, (NT if m + 1 == MB else (m + 1) * mb)
            idx = perm[e * NT + lo:e * NT + hi]
            n = hi - lo
            tup = ref_call(cpu, "lean_ffi_gather_minibatch", VP, FA(k["obs"]), FA(k["acts"]), FA(k["adv"]),
                           FA(k["rets"]), FA(k["olps"]), FA(idx), n, D)
            mbObs = arr(O.ctor_field(tup, 0))
            t2 = O.ctor_field(tup, 1)
            mbAct = arr(O.ctor_field(t2, 0))
            t3 = O.ctor_field(t2, 1)
            mbAdv = arr(O.ctor_field(t3, 0))
            t4 = O.ctor_field(t3, 1)
            mbRet, mbOlp = arr(O.ctor_field(t4, 0)), arr(O.ctor_field(t4, 1))
            advN = arr(ref_call(cfb, "lean_cuda_adv_normalize", VP, FA(mbAdv), n))
            g = arr(ref_call(cpu, "lean_ffi_mlp_ppo_grad_batch_blas", VP, FA(pm[:k["P"]]), FA(mbObs), FA(mbAct),
                             FA(advN), FA(mbRet), FA(mbOlp), n, H, D, A, k["vf"], k["ent"], k["clip"]))
            pm = arr(ref_call(cpu, "lean_ffi_muon_step_mlp", VP, FA(pm), FA(g), H, D, A + 1, 1.0 / n, k["lr"],
                              k["wd"], k["mu"], k["eps"]))
    np.savez(os.path.join(OUT, "train_update.npz"), out=pm, perm=perm,
             **{x: k[x] for x in ("pm0", "obs", "acts", "adv", "rets", "olps")},
             meta=np.array([NT, D, H, A, E, MB, k["vf"], k["ent"], k["clip"], k["lr"], k["wd"], k["mu"], k["eps"],
                            k["perm_seed"]]))

    # host bookkeeping twins: shuffle, GAE, prioritized sampling, gather
    shuf = {}
    for i, (NT_, E_, seed) in enumerate([(48, 3, 0x1234), (1000, 2, 0xFEEDFACE12345678), (1, 1, 7)]):
        shuf[f"perm{i}"] = arr(ref_call(cpu, "lean_ffi_shuffle_perm", VP, NT_, E_, ("u64", seed)))
        shuf[f"args{i}"] = np.array([NT_, E_, seed], dtype=np.uint64)
    np.savez(os.path.join(OUT, "shuffle.npz"), **shuf)

    rng = kat.Rng(0x6AE)
    N, T = 16, 20
    vals = np.array([rng.randF(-2.0, 2.0) for _ in range(N * T)])
    rews = np.array([rng.randF(-1.5, 1.5) for _ in range(N * T)])
    terms = np.array([1.0 if rng.randF(0.0, 1.0) < 0.1 else 0.0 for _ in range(N * T)])
    ga = arr(ref_call(cpu, "lean_ffi_gae_soa", VP, FA(vals), FA(rews), FA(terms), N, T, 0.995, 0.90))
    np.savez(os.path.join(OUT, "gae.npz"), vals=vals, rews=rews, terms=terms, out=ga, meta=np.array([N, T, 0.995, 0.9]))

    rng = kat.Rng(0x9F10)
    N, mbSegs = 200, 64
    L1 = np.array([rng.randF(0.0, 30.0) for _ in range(N)])
    pr = ref_call(cpu, "lean_ffi_prio_sample", VP, FA(L1), N, 64, mbSegs, 0.8, 0.2, ("u64", 0xABCDEF))
    np.savez(os.path.join(OUT, "prio.npz"), L1=L1, idx=arr(O.ctor_field(pr, 0)), mbPrio=arr(O.ctor_field(pr, 1)),
             meta=np.array([N, 64, mbSegs, 0.8, 0.2, 0xABCDEF], dtype=np.float64))
    # MinGRU: the per-sequence BPTT gradient (verify-mingru-grad-gpu inputs), the minibatch scalar gather,
    # and one whole update composed from the reference's own C pieces
    k = kat.kat_mingru_grad()
    s = k["seqs"]
    per = []
    for b in range(k["B"]):
        per.append(arr(ref_call(cpu, "lean_ffi_mingru_ppo_grad_seq", VP, FA(k["params"]), FA(s["obs"][b]),
                                FA(s["act"][b]), FA(s["adv"][b]), FA(s["ret"][b]), FA(s["old"][b]), FA(s["term"][b]),
                                FA(s["ov"][b]), k["T"], k["H"], k["D"], k["L"], k["A"], k["vf"], k["ent"], k["clip"],
                                k["vfClip"])))
    np.savez(os.path.join(OUT, "mingru_grad.npz"), params=k["params"], obsTB=k["obsTB"], scal=k["scal"],
             seq0=per[0], seq1=per[1],
             meta=np.array([k["D"], k["H"], k["L"], k["A"], k["T"], k["B"], k["vf"], k["ent"], k["clip"],
                            k["vfClip"]]))

    rng = kat.Rng(0x6A7)
    N, T, D, Bmb = 10, 5, 3, 7
    cols = {x: np.array([rng.randF(-1.0, 1.0) for _ in range(N * T)]) for x in ("adv", "value", "logp")}
    cols["act"] = np.array([float(rng.next() % 4) for _ in range(N * T)])
    cols["term"] = np.array([1.0 if rng.randF(0.0, 1.0) < 0.2 else 0.0 for _ in range(N * T)])
    seg = np.array([float(rng.next() % N) for _ in range(Bmb)])
    mbp = np.array([rng.randF(0.2, 1.5) for _ in range(Bmb)])
    obsCol = np.zeros(N * T * D)
    g = arr(ref_call(cpu, "lean_ffi_gather_seq_minibatch", VP, FA(obsCol), FA(cols["act"]), FA(cols["logp"]),
                     FA(cols["term"]), FA(cols["adv"]), FA(cols["value"]), FA(seg), FA(mbp), T, Bmb, D, N))
    np.savez(os.path.join(OUT, "gather_seq.npz"), out=g, seg=seg, mbPrio=mbp, meta=np.array([N, T, D, Bmb]), **cols)

    k = kat.kat_mingru_update()
    N, T, D, H, L, A, K = (k[x] for x in ("N", "T", "D", "H", "L", "A", "K"))
    P = O.mg_param_count(D, H, L, A, K)
    pm = k["pm0"].copy()
    value, ratio = k["val0"].copy(), np.ones(N * T)
    r = k["rng"]
    Bmb = k["mbSegs"]
    for _ in range(k["numMB"]):
        adv = arr(ref_call(cfb, "lean_cuda_vtrace_mingru", VP, FA(k["rew"]), FA(value), FA(k["term"]), FA(ratio),
                           FA(k["boot"]), N, T, k["gamma"], k["lam"], k["rho"], k["c"]))
        l1 = O.adv_l1(adv, N, T)
        pr = ref_call(cpu, "lean_ffi_prio_sample", VP, FA(l1), N, T, Bmb, k["alpha"], k["beta"], ("u64", r))
        seg, mbp = arr(O.ctor_field(pr, 0)), arr(O.ctor_field(pr, 1))
        r = (r + Bmb * kat.GOLD) & kat.M64
        sc = arr(ref_call(cpu, "lean_ffi_gather_seq_minibatch", VP, FA(np.zeros(N * T * D)), FA(k["act"]),
                          FA(k["logp"]), FA(k["term"]), FA(adv), FA(value), FA(seg), FA(mbp), T, Bmb, D, N))
        nb = T * Bmb
        g = np.zeros(P)
        newlp, newval = np.zeros(nb), np.zeros(nb)
        for b in range(Bmb):
            e = int(seg[b])
            obs_seq = k["obs"][e * T * D:(e + 1) * T * D]
            cs = [sc[q * nb + b:(q + 1) * nb:Bmb] for q in range(6)]
            gs = arr(ref_call(cpu, "lean_ffi_mingru_ppo_grad_seq", VP, FA(pm[:P]), FA(obs_seq), *[FA(x) for x in cs],
                              T, H, D, L, A, k["vf"], k["ent"], k["clip"], k["vfClip"]))
            g = g + gs[:P]
            newlp[b::Bmb] = gs[P:P + T]
            newval[b::Bmb] = gs[P + T:]
        for b in range(Bmb):
            e = int(seg[b])
            for t in range(T):
                ratio[e * T + t] = np.exp(newlp[t * Bmb + b] - k["logp"][e * T + t])
                value[e * T + t] = newval[t * Bmb + b]
        gc = O.grad_clip(g, k["maxGradNorm"], 1.0 / nb)
        off = 0
        shapes = [(H, D, H)] + [(K * H, H, 0)] * L + [(A, H, A), (1, H, 1)]
        for rows, cols_, nbias in shapes:
            n = rows * cols_
            o = arr(ref_call(cfb, "lean_cuda_muon_stepmat", VP, FA(pm[off:off + n]), FA(gc[off:off + n]),
                             FA(pm[P + off:P + off + n]), rows, cols_, k["lr"], k["wd"], k["mu"], k["eps"]))
            pm[off:off + n], pm[P + off:P + off + n] = o[:n], o[n:]
            off += n
            if nbias:
                nb_, nm_ = np.zeros(nbias), np.zeros(nbias)
                O.orc().orc_muon_stepvec(O._ptr(pm[off:off + nbias].copy()), O._ptr(gc[off:off + nbias].copy()),
                                         O._ptr(pm[P + off:P + off + nbias].copy()), nbias, k["lr"], k["wd"], k["mu"],
                                         O._ptr(nb_), O._ptr(nm_))
                pm[off:off + nbias], pm[P + off:P + off + nbias] = nb_, nm_
                off += nbias
    np.savez(os.path.join(OUT, "mingru_update.npz"), out=pm, rng_out=np.array([r], dtype=np.uint64))

    # Gaussian (continuous) head: out = [means | log-stds | value], O = 2W+1. The bias of the log-std rows
    # puts some raw log-stds above the clamp's upper end 2 (their gradient is cut); none reaches the CPU
    # form's lower end -5, below which the CPU (-5) and device (-20) clamps differ.
    g = np.random.default_rng(0x6A055)
    N, D, H, W = 37, 7, 24, 3
    Og = 2 * W + 1
    P = H * D + H + Og * H + Og
    params = g.uniform(-0.25, 0.25, P)
    params[H * D + H + Og * H + W:H * D + H + Og * H + 2 * W] = [-0.5, 0.3, 2.05]
    obs, acts = g.uniform(-1, 1, N * D), g.standard_normal(N * W)
    advs, rets, olps = g.standard_normal(N), g.standard_normal(N), g.uniform(-5.0, -1.0, N)
    ov = rets + 0.3 * g.standard_normal(N)
    ins = dict(params=params, obs=obs, acts=acts, advs=advs, rets=rets, olps=olps, ov=ov)
    base = (FA(params), FA(obs), FA(acts), FA(advs), FA(rets), FA(olps))
    g_plain = arr(ref_call(cpu, "lean_ffi_gauss_ppo_grad_batch", VP, *base, N, H, D, W, 0.5, 0.01, 0.2))
    base = (FA(params), FA(obs), FA(acts), FA(advs), FA(rets), FA(olps), FA(ov))
    g_vc = arr(ref_call(cpu, "lean_ffi_gauss_ppo_grad_batch_vclip", VP, *base, N, H, D, W, 0.5, 0.01, 0.2, 0.2))
    np.savez(os.path.join(OUT, "gauss_grad.npz"), g_plain=g_plain, g_vclip=g_vc,
             meta=np.array([N, D, H, W, 0.5, 0.01, 0.2, 0.2]), **ins)

    # A whole Gaussian-head update (2 epochs x 4 minibatches, value clip on, no norm clip) composed from the
    # reference's C: gather, adv normalisation, the Gaussian gradient, lean_ffi_muon_step_mlp with 1/n.
    NT, E, MB = 64, 2, 4
    pm0 = np.concatenate([params, g.uniform(-0.01, 0.01, P)])
    obsT, actsT = g.uniform(-1, 1, NT * D), g.standard_normal(NT * W)
    advT, retT, olpT = g.standard_normal(NT), g.standard_normal(NT), g.uniform(-5.0, -1.0, NT)
    ovT = retT + 0.3 * g.standard_normal(NT)
    perm = arr(ref_call(cpu, "lean_ffi_shuffle_perm", VP, NT, E, ("u64", 0x5EED)))
    hyp = dict(lr=0.01, wd=0.001, mu=0.95, eps=1e-7, vf=0.5, ent=0.01, clip=0.2, vfClip=0.2)
    pm = pm0.copy()
    mb = NT // MB
    for e in range(E):
        for m in range(MB):
            lo, hi = m * mb, (NT if m + 1 == MB else (m + 1) * mb)
            idx = perm[e * NT + lo:e * NT + hi].astype(np.int64)
            n = idx.size
            mObs = obsT.reshape(NT, D)[idx].ravel()
            mAct = actsT.reshape(NT, W)[idx].ravel()
            advN = arr(ref_call(cfb, "lean_cuda_adv_normalize", VP, FA(advT[idx]), n))
            gg = arr(ref_call(cpu, "lean_ffi_gauss_ppo_grad_batch_vclip", VP, FA(pm[:P]), FA(mObs), FA(mAct),
                              FA(advN), FA(retT[idx]), FA(olpT[idx]), FA(ovT[idx]), n, H, D, W, hyp["vf"],
                              hyp["ent"], hyp["clip"], hyp["vfClip"]))
            pm = arr(ref_call(cpu, "lean_ffi_muon_step_mlp", VP, FA(pm), FA(gg[:P]), H, D, Og, 1.0 / n, hyp["lr"],
                              hyp["wd"], hyp["mu"], hyp["eps"]))
    np.savez(os.path.join(OUT, "gauss_update.npz"), pm0=pm0, out=pm, obs=obsT, acts=actsT, adv=advT, ret=retT,
             olp=olpT, ov=ovT, perm=perm, meta=np.array([NT, D, H, W, E, MB]),
             hyp=np.array([hyp[x] for x in ("lr", "wd", "mu", "eps", "vf", "ent", "clip", "vfClip")]))

    # LSTM: three sequences of the reference's scalar BPTT gradient (lean_ffi_lstm_ppo_grad_seq) from
    # detached non-zero initial states, a terminal mid-sequence; and its GAE + normalisation
    # (lean_ffi_lstm_gae_boot_norm) on time-major columns.
    g = np.random.default_rng(0x157)
    T, H, D, A, B = 9, 6, 5, 4, 3
    P = 4 * H * D + 4 * H * H + 4 * H + (A + 1) * H + (A + 1)
    lp = g.uniform(-0.4, 0.4, P)
    obsB = g.standard_normal(T * B * D)
    actB = g.integers(0, A, T * B).astype(float)
    advB, retB, olpB = g.standard_normal(T * B), g.standard_normal(T * B), g.uniform(-3, -0.5, T * B)
    termB = (g.random(T * B) < 0.15).astype(float)
    h0s, c0s = g.uniform(-0.5, 0.5, B * H), g.uniform(-0.5, 0.5, B * H)
    seqs = []
    for b in range(B):
        rows = [t * B + b for t in range(T)]
        o = np.concatenate([obsB[r * D:(r + 1) * D] for r in rows])
        seqs.append(arr(ref_call(cpu, "lean_ffi_lstm_ppo_grad_seq", VP, FA(lp), FA(o), FA(actB[rows]),
                                 FA(advB[rows]), FA(retB[rows]), FA(olpB[rows]), FA(termB[rows]),
                                 FA(h0s[b * H:(b + 1) * H]), FA(c0s[b * H:(b + 1) * H]), T, H, D, A, 0.5, 0.01,
                                 0.2)))
    N = 7
    vals, rews = g.standard_normal(N * T), g.standard_normal(N * T)
    terms, boot = (g.random(N * T) < 0.2).astype(float), g.standard_normal(N)
    gae = arr(ref_call(cpu, "lean_ffi_lstm_gae_boot_norm", VP, FA(vals), FA(rews), FA(terms), FA(boot), N, T, 0.99,
                       0.95))
    np.savez(os.path.join(OUT, "lstm.npz"), params=lp, obsB=obsB, actB=actB, advB=advB, retB=retB, olpB=olpB,
             termB=termB, h0s=h0s, c0s=c0s, seqs=np.stack(seqs), meta=np.array([T, H, D, A, B]), vals=vals, rews=rews,
             terms=terms, boot=boot, gae=gae, gae_meta=np.array([N, T, 0.99, 0.95]))
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
