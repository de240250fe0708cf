"""Regenerate the golden fixtures in tests/golden/ from the reference's own compiled C.

Run in the build container (the reference tree must be present and no GPU visible):

    make -C oracle all ref && python tests/golden/gen_golden.py

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


def main():
    cpu = O.ref_cpu()
    cfb = O.ref_cudafb()
    out = {}

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
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
