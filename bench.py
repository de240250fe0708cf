#!/usr/bin/env python
"""PPO+Muon update throughput on B200 (the north-star metric of BASELINE.json).

One step = one whole PPO+Muon update of the C5 large-MLP policy: the
advantage scan over the rollout columns, then 4 epochs x 16 minibatches of 262,144 rows, each
minibatch = gather, forward (obs 1024 -> 5 x 2048 GELU -> 64 logits + value), PPO objective
gradient, backward, grad-norm clip, Muon (Newton-Schulz) on every weight matrix. Inputs are seeded
synthetic rollout columns already resident in HBM (obs 17 GB fp32 > L2, so no flush is needed).

value    samples/s = world x N_envs x horizon / device time of one update (max over ranks)
e2e      the same update through the reference-facing C-ABI call (pl_train_update_resident) from
         pinned HOST buffers, with the host GAE and shuffle, H2D copies and the params[0] read-back
         inside the timed region
roofline the tcgen05 GEMM kernels of the step (forward, PPO head, data and weight gradients),
         timed live with CUDA events on the launch stream; achieved = algorithmic flops / time
cpu_baseline  the CPU restatement (oracle/cpu_port.py, numpy f64 on all host cores) on a bounded
         sample, scaled to one update

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c5|c1]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "PPO+Muon update samples/sec at 1/2/4/8 B200; NS/GEMM % tensor peak"
QUINTIC = [(3.4445, -4.7750, 2.0315)] * 5

WORKLOADS = {
    # 65536 envs x 64, obs 1024, 4 hidden 2048 (+ the 1024->2048 encoder), 64 actions
    "c5": dict(name="C5 large-MLP PPO+Muon update (configs[4])", N=65536, T=64, D=1024, H=2048, L=5, A=64, act=1,
               Nmb=262144, epochs=4, obs="normal", rew="normal", done=0.01, lr=0.02),
    # profiling case of C5: the same per-row shapes, 1024 envs, one minibatch of 65,536 rows
    "c5p": dict(name="C5 per-row shapes, 1024 envs (profiling case)", N=1024, T=64, D=1024, H=2048, L=5, A=64,
                act=1, Nmb=65536, epochs=1, obs="normal", rew="normal", done=0.01, lr=0.02),
    # CartPole-shaped, 1024 envs x 64, obs 4, hidden 128, 2 actions, fp32. The network
    # is the reference's own (ReLU; its CPU path has no GELU) so the reference arm runs the same work through its
    # compiled C; no value clip (lean_ffi_mlp_ppo_grad_batch_blas has none)
    "c1": dict(name="C1 CartPole-shaped PPO+Muon update (configs[0], the reference's ReLU network, fp32)", N=1024,
               T=64, D=4, H=128, L=1, A=2, act=0, Nmb=16384, epochs=4, obs="normal", rew="bern", done=0.01, lr=0.02,
               bf16=0, vfclip=0.0, maxgn=1.5),
}


class Arch(C.Structure):
    _fields_ = [("L", C.c_size_t), ("act", C.c_int), ("ns_coeffs", C.POINTER(C.c_double)), ("ns_iters", C.c_size_t)]


class Desc(C.Structure):
    _fields_ = [("NT", C.c_size_t), ("D", C.c_size_t), ("H", C.c_size_t), ("A", C.c_size_t), ("epochs", C.c_size_t),
                ("numMB", C.c_size_t), ("arch", Arch), ("wd", C.c_double), ("mu", C.c_double), ("eps", C.c_double),
                ("vfCoef", C.c_double), ("entCoef", C.c_double), ("clipEps", C.c_double), ("vfClip", C.c_double),
                ("maxGradNorm", C.c_double), ("bf16", C.c_uint8), ("use_old_values", C.c_uint8), ("rank", C.c_int),
                ("world", C.c_int), ("comm", C.c_void_p)]


# DRAM bytes per launch of the roofline kernel set (forward, PPO-head, data- and weight-gradient
# tc_gemm launches), from one ncu capture of every GEMM launch of a 65,536-row update
# (profiles/tc_gemm_dram_c5p.md: 11,464 MB over the 17 launches of one minibatch), scaled x4 to the
# 262,144-row minibatch of configs[4] (every one of these launches moves bytes in proportion to rows).
C5_GEMM_DRAM_BYTES_PER_LAUNCH = 4 * 11464e6 / 17


def c5_gemm_algorithmic_bytes_per_launch(Nmb, D, H, L, A):
    """Bytes each launch of one minibatch must move at least (bf16 activations read once, outputs written
    once, weights read once), averaged over the 3L + 2 launches of the roofline kernel set."""
    Op = 128 if A + 1 > 64 else 64
    act = Nmb * H * 2
    fwd = (Nmb * D * 2 + 2 * act) + (L - 1) * (act + 2 * act) + (act + Nmb * Op * 2)
    dgrad = (L - 1) * 3 * act + (Nmb * Op * 2 + act + act)
    wgrad = (Nmb * D * 2 + act) + (L - 1) * 2 * act + (Nmb * Op * 2 + act)
    return (fwd + dgrad + wgrad) / (3 * L + 2)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops_sustained", d.get("bf16_tflops")), d.get("hbm_gbs"), "measured"
    return 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def xavier_pm(D, H, A, L, seed):
    g = np.random.default_rng(seed)
    P = H * D + H + (L - 1) * (H * H + H) + (A + 1) * H + A + 1
    pm = np.zeros(2 * P)
    off = 0
    for l in range(L + 1):
        fin = D if l == 0 else H
        fout = A + 1 if l == L else H
        lim = np.sqrt(6.0 / (fin + fout))
        pm[off:off + fout * fin] = g.uniform(-lim, lim, fout * fin)
        off += fout * fin + fout
    return P, pm


def check(rc, L):
    if rc != 0:
        raise RuntimeError(L.pl_last_error().decode())


def make_comm(L, rank, world):
    """NCCL communicator of the library (one per rank); the 128-byte id travels over the
    torch.distributed process group (plumbing only)."""
    import torch

    if world == 1:
        return None
    ident = (C.c_uint8 * 128)()
    if rank == 0:
        check(L.pl_comm_unique_id(ident), L)
    t = torch.tensor(list(bytes(ident)), dtype=torch.uint8, device="cuda")
    torch.distributed.broadcast(t, 0)
    ident = (C.c_uint8 * 128)(*t.cpu().tolist())
    comm = C.c_void_p()
    L.pl_comm_create.argtypes = [C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]
    check(L.pl_comm_create(rank, world, ident, C.byref(comm)), L)
    return comm


def run_ours(args, wl, rank, world, local_rank, comm=None):
    import torch

    import pufferlean_b200 as plb

    torch.cuda.set_device(local_rank)
    L = plb.lib()
    check(L.pl_set_device(local_rank), L)
    dp = C.POINTER(C.c_double)
    vp = C.c_void_p
    L.pl_update_create.argtypes = [C.c_size_t, C.POINTER(Desc), C.POINTER(vp)]
    L.pl_update_set_columns_dev.argtypes = [vp] * 9
    L.pl_update_set_advantages_dev.argtypes = [vp] * 5 + [C.c_size_t] + [C.c_double] * 4 + [vp]
    L.pl_update_run.argtypes = [vp, C.c_double, vp]
    L.pl_update_profile.argtypes = [vp, C.c_int]
    L.pl_update_profile_read.argtypes = [vp, dp, dp, dp]
    L.pl_update_destroy.argtypes = [vp]

    N, T, D, H, Lh, A = wl["N"], wl["T"], wl["D"], wl["H"], wl["L"], wl["A"]
    NT = N * T
    Nmb, E = wl["Nmb"], wl["epochs"]
    numMB = NT // Nmb
    strong = getattr(args, "scaling", "weak") == "strong"
    seed = 1234 + (0 if strong else rank)  # strong scaling: every rank holds the same rollout
    gen = torch.Generator(device="cuda").manual_seed(seed)
    obs = torch.randn(NT, D, device="cuda", generator=gen) if wl["obs"] == "normal" else \
        torch.rand(NT, D, device="cuda", generator=gen)
    acts = torch.randint(0, A, (NT,), device="cuda", generator=gen).double()
    rew = torch.randn(NT, device="cuda", generator=gen) if wl["rew"] == "normal" else \
        (torch.rand(NT, device="cuda", generator=gen) < 0.5).float()
    val = torch.randn(NT, device="cuda", generator=gen)
    term = (torch.rand(NT, device="cuda", generator=gen) < wl["done"]).float()
    olp = (torch.full((NT,), float(np.log(1.0 / A)), device="cuda", dtype=torch.float64) +
           0.05 * torch.randn(NT, device="cuda", generator=gen, dtype=torch.float64))
    perm_h = plb.shuffle_perm(NT, E, 0xC5 + (0 if strong else rank))
    perm = torch.from_numpy(perm_h).cuda()
    P, pm = xavier_pm(D, H, A, Lh, 42)
    handle = plb.policy_load(pm, P)
    co = np.ascontiguousarray(np.array(QUINTIC, dtype=np.float64))
    if comm is None:
        comm = make_comm(L, rank, world)
    desc = Desc(NT=NT, D=D, H=H, A=A, epochs=E, numMB=numMB, arch=Arch(Lh, wl["act"], co.ctypes.data_as(dp), 5),
                wd=0.0, mu=0.95, eps=1e-12, vfCoef=0.5, entCoef=0.01, clipEps=0.2, vfClip=wl.get("vfclip", 0.2),
                maxGradNorm=wl.get("maxgn", 1.5), bf16=wl.get("bf16", 1), use_old_values=int(wl.get("vfclip", 0.2) > 0),
                rank=rank, world=world, comm=comm)
    u = vp()
    check(L.pl_update_create(handle, C.byref(desc), C.byref(u)), L)
    if strong and world > 1:
        L.pl_update_split_minibatch.argtypes = [vp, C.c_int]
        check(L.pl_update_split_minibatch(u, 1), L)
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        check(L.pl_update_set_columns_dev(u, obs.data_ptr(), acts.data_ptr(), None, None, olp.data_ptr(), None,
                                          perm.data_ptr(), stream), L)
        check(L.pl_update_set_advantages_dev(u, rew.data_ptr(), val.data_ptr(), term.data_ptr(), None, T, 0.995, 0.90,
                                             1.0, 1.0, stream), L)
        check(L.pl_update_run(u, wl["lr"], stream), L)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    l0 = L.pl_kernel_launch_count()
    # inputs smaller than L2 are timed step by step with a 256 MB write between steps, so
    # every step starts with a cold L2; larger ones (configs[4]: 17 GB of observations) need no flush
    in_bytes = NT * (D + 8) * 4
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda") if in_bytes < (256 << 20) else None
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps if flush is not None else 1)]
    with ClockSampler(local_rank) as clk:
        if flush is None:
            evs[0][0].record()
            for _ in range(args.steps):
                step()
            evs[0][1].record()
        else:
            for e0, e1 in evs:
                flush.fill_(1.0)
                e0.record()
                step()
                e1.record()
        torch.cuda.synchronize()
    launches = L.pl_kernel_launch_count() - l0
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / args.steps
    # the per-class breakdown (CUDA events around each launch group) comes from untimed steps after the
    # timed ones, so that no profiling event sits inside the timed region
    psteps = min(args.steps, 2)
    if world > 1:
        torch.distributed.barrier()
    check(L.pl_update_profile(u, 1), L)
    for _ in range(psteps):
        if flush is not None:
            flush.fill_(1.0)
        step()
    torch.cuda.synchronize()
    pms, pfl, pln = (C.c_double * 8)(), (C.c_double * 8)(), (C.c_double * 8)()
    check(L.pl_update_profile_read(u, pms, pfl, pln), L)
    cms, cbytes, cn = C.c_double(), C.c_double(), C.c_double()
    L.pl_update_comm_profile_read.argtypes = [vp, dp, dp, dp]
    check(L.pl_update_comm_profile_read(u, C.byref(cms), C.byref(cbytes), C.byref(cn)), L)
    check(L.pl_update_profile(u, 0), L)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = (1 if strong else world) * NT / (ms / 1e3)
    peak_tf, peak_hbm, peak_kind = peaks()
    gemm_ms = sum(pms[i] for i in range(4))
    gemm_fl = sum(pfl[i] for i in range(4))
    gemm_n = sum(pln[i] for i in range(4))
    achieved = gemm_fl / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
    ns_tf = pfl[4] / (pms[4] / 1e3) / 1e12 if pms[4] > 0 else 0.0
    prof = {k: {"ms_per_step": pms[i] / psteps, "tflops": (pfl[i] / (pms[i] / 1e3) / 1e12) if pms[i] > 0 and
                pfl[i] > 0 else None, "launches_per_step": pln[i] / psteps}
            for i, k in enumerate(["fwd_gemm", "ppo_head_gemm", "dgrad_gemm", "wgrad_gemm", "newton_schulz",
                                   "gather_stats", "optimizer_elementwise", "dp_collectives"])}
    L.pl_update_destroy(u)
    del obs
    torch.cuda.empty_cache()

    out = {
        "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if strong and world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16" if wl.get("bf16", 1) else "f32",
        "data": "synthetic (seeded; obs N(0,1), rewards %s, dones Bern(%g))" % (
            "N(0,1)" if wl["rew"] == "normal" else "Bern(0.5)", wl["done"]),
        "config": {"workload": wl["name"], "N_envs_per_gpu": N, "horizon": T, "obs_dim": D, "hidden": H,
                   "hidden_layers": Lh, "actions": A, "activation": "gelu" if wl["act"] else "relu",
                   "minibatch_rows_per_gpu": Nmb // world if strong else Nmb, "epochs": E,
                   "minibatches_per_epoch": numMB,
                   "ns_coeffs": "quintic (3.4445,-4.7750,2.0315) x5", "params": P,
                   "l2": ("no flush: the obs column alone (fp32 %.1f GB) exceeds L2" % (NT * D * 4 / 1e9)
                          if flush is None else "L2 flushed (256 MB write) before each timed step"),
                   "parallelism": f"dp{world}" + (" (one rollout, each minibatch split over the ranks)"
                                                   if strong and world > 1 else "")},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": achieved / peak_tf if peak_tf else None,
                     "traffic": C5_GEMM_DRAM_BYTES_PER_LAUNCH if wl is WORKLOADS["c5"] else None,
                     "traffic_algorithmic": c5_gemm_algorithmic_bytes_per_launch(Nmb, D, H, Lh, A),
                     "traffic_source": "ncu dram__bytes_read+write of every GEMM launch of a 65,536-row update, x4 "
                                       "to 262,144 rows (profiles/tc_gemm_dram_c5p.md)",
                     "kernel": "tc_gemm_kernel (all forward/PPO-head/dgrad/wgrad launches of the step)",
                     "launches_per_step": gemm_n / psteps, "peak_kind": peak_kind + " (bf16 sustained)"},
        "newton_schulz": {"tflops": ns_tf, "frac": ns_tf / peak_tf if peak_tf else None,
                          "ms_per_step": pms[4] / psteps},
        "profile": prof,
        "profile_how": "CUDA events around each launch group, recorded in %d untimed step(s) after the timed ones" % psteps,
        "gpu_launches": int(launches),
        "dp_allreduce": None if world == 1 else {
            "ms_per_step_on_comm_stream": cms.value / psteps,
            "ms_per_step_exposed": pms[7] / psteps,
            "bytes_per_rank_per_step": cbytes.value / psteps,
            "launches_per_step": cn.value / psteps,
            "bus_gbs": (cbytes.value * 2 * (world - 1) / world / (cms.value / 1e3) / 1e9) if cms.value > 0 else None,
            "how": "per-layer fp32 ncclAllReduce on a second stream, each started when its layer's gradient is "
                   "complete; bus GB/s = bytes x 2(N-1)/N / time on that stream"},
        "clocks": clk.summary(),
    }
    return out, dict(handle=handle, P=P, pm=pm, comm=comm, desc=desc, co=co)


def run_e2e(args, wl, state, rank, world, local_rank):
    """The same update through pl_train_update_resident with pinned host buffers: host GAE and
    shuffle (the reference's per-update host C), H2D of the f64 columns, the update, the 8-byte
    params[0] read-back."""
    import torch

    import pufferlean_b200 as plb

    N, T, D, H, Lh, A = wl["N"], wl["T"], wl["D"], wl["H"], wl["L"], wl["A"]
    NT = N * T
    E, Nmb = wl["epochs"], wl["Nmb"]
    numMB = NT // Nmb
    strong = getattr(args, "scaling", "weak") == "strong"
    gen = torch.Generator(device="cuda").manual_seed(99 + (0 if strong else rank))
    obs_h = torch.empty(NT * D, dtype=torch.float64, pin_memory=True)
    chunk = 1 << 27
    for o in range(0, NT * D, chunk):
        n = min(chunk, NT * D - o)
        obs_h[o:o + n].copy_(torch.randn(n, device="cuda", generator=gen, dtype=torch.float64))
    g = np.random.default_rng(7 + (0 if strong else rank))
    cols = {k: torch.empty(NT, dtype=torch.float64, pin_memory=True) for k in ("acts", "olp", "val", "rew", "term")}
    cols["acts"].copy_(torch.from_numpy(g.integers(0, A, NT).astype(np.float64)))
    cols["olp"].copy_(torch.from_numpy(np.log(1.0 / A) + 0.05 * g.standard_normal(NT)))
    cols["val"].copy_(torch.from_numpy(g.standard_normal(NT)))
    cols["rew"].copy_(torch.from_numpy(g.standard_normal(NT)))
    cols["term"].copy_(torch.from_numpy((g.random(NT) < wl["done"]).astype(np.float64)))
    gae = torch.empty(2 * NT, dtype=torch.float64, pin_memory=True)
    perm = torch.empty(E * NT, dtype=torch.float64, pin_memory=True)
    L = plb.lib()
    dp = C.POINTER(C.c_double)
    L.pl_train_update_resident_deep.argtypes = ([C.c_size_t, C.POINTER(Arch)] + [dp] * 6 + [C.c_size_t, dp] +
                                                [C.c_size_t] * 6 + [C.c_double] * 9 + [C.c_uint8, dp])
    L.pl_gae_soa.argtypes = [dp] * 3 + [C.c_size_t, C.c_size_t, C.c_double, C.c_double, dp]
    L.pl_shuffle_perm.argtypes = [C.c_size_t, C.c_size_t, C.c_uint64, dp]
    co = np.ascontiguousarray(np.array(QUINTIC, dtype=np.float64))
    arch = Arch(Lh, wl["act"], co.ctypes.data_as(dp), 5)
    out0 = np.zeros(1)

    def P_(t):
        return C.cast(t.data_ptr(), dp)

    def step(i):
        check(L.pl_gae_soa(P_(cols["val"]), P_(cols["rew"]), P_(cols["term"]), N, T, 0.995, 0.90, P_(gae)), L)
        check(L.pl_shuffle_perm(NT, E, 0xE2E + i, P_(perm)), L)
        adv = C.cast(gae.data_ptr(), dp)
        ret = C.cast(gae.data_ptr() + 8 * NT, dp)
        check(L.pl_train_update_resident_deep(state["handle"], C.byref(arch), P_(obs_h), P_(cols["acts"]), adv, ret,
                                              P_(cols["olp"]), P_(cols["val"]), NT, P_(perm), NT, D, H, A, E, numMB,
                                              wl["lr"], 0.0, 0.95, 1e-12, 0.5, 0.01, 0.2, wl.get("vfclip", 0.2),
                                              wl.get("maxgn", 1.5), wl.get("bf16", 1), out0.ctypes.data_as(dp)), L)

    if world > 1:
        # the reference's C-ABI is single-GPU; the data-parallel form of the same call is the session
        # API fed from the same pinned host columns
        vp = C.c_void_p
        L.pl_update_create.argtypes = [C.c_size_t, C.POINTER(Desc), C.POINTER(vp)]
        L.pl_update_run_columns.argtypes = [vp] * 8 + [C.c_double, vp]
        L.pl_update_destroy.argtypes = [vp]
        sess = vp()
        check(L.pl_update_create(state["handle"], C.byref(state["desc"]), C.byref(sess)), L)
        strong = getattr(args, "scaling", "weak") == "strong"
        if strong:
            L.pl_update_split_minibatch.argtypes = [vp, C.c_int]
            check(L.pl_update_split_minibatch(sess, 1), L)

        def step(i):  # noqa: F811
            check(L.pl_gae_soa(P_(cols["val"]), P_(cols["rew"]), P_(cols["term"]), N, T, 0.995, 0.90, P_(gae)), L)
            check(L.pl_shuffle_perm(NT, E, 0xE2E + (0 if strong else 1000 * rank) + i, P_(perm)), L)
            check(L.pl_update_run_columns(sess, obs_h.data_ptr(), cols["acts"].data_ptr(), gae.data_ptr(),
                                          gae.data_ptr() + 8 * NT, cols["olp"].data_ptr(), cols["val"].data_ptr(),
                                          perm.data_ptr(), wl["lr"], None), L)
            cudart_memcpy_d2h(out0, state["handle"])  # synchronizes, then reads params[0]
    step(0)
    if world > 1:
        torch.distributed.barrier()
    k = max(1, min(args.steps, 3))
    t0 = time.perf_counter()
    for i in range(k):
        step(i + 1)
    dt = (time.perf_counter() - t0) / k
    if world > 1:
        t = torch.tensor([dt], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dt = float(t.item())
    if world > 1:
        L.pl_update_destroy(sess)
    # the bytes the library copied in the last update: observations partly as bf16 rows rounded on the
    # host threads, partly as f64 rows converted on the device; the other columns and the shuffle
    L.pl_update_last_upload_bytes.restype = C.c_uint64
    h2d = int(L.pl_update_last_upload_bytes())
    return {"value": (1 if strong else world) * NT / dt, "unit": "samples/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": 8 if world == 1 else 16,
            "steps": k, "s_per_step": dt,
            "path": ("pl_train_update_resident_deep (the reference-facing C-ABI call)" if world == 1 else
                     "pl_update_run_columns on a data-parallel session (the C-ABI's DP form)") +
                    ", pinned host f64 columns, host GAE + shuffle in the timed region"}


def measure_vtrace_c2(reps=20):
    """the fp32 V-trace scan over 4096 segments x 64, 20 B per element
    (rewards, values, dones, importance ratios in; advantages out). One set is 5.2 MB and would sit
    in L2, so 64 rotating sets (335 MB) are scanned back to back, each by its own launch inside one
    CUDA graph; the single-set latency is reported beside it."""
    import torch

    import pufferlean_b200 as plb

    L = plb.lib()
    B, T, S = 4096, 64, 64
    g = torch.Generator(device="cuda").manual_seed(2)
    rew = torch.rand(S, B * T, device="cuda", generator=g) * 2 - 1
    val = torch.randn(S, B * T, device="cuda", generator=g)
    term = (torch.rand(S, B * T, device="cuda", generator=g) < 0.01).float()
    imp = torch.exp(0.1 * torch.randn(S, B * T, device="cuda", generator=g))
    adv = torch.empty(S, B * T, device="cuda")
    st = torch.cuda.Stream()

    def one(i, stream):
        rc = L.pl_vtrace_f32_dev(rew[i].data_ptr(), val[i].data_ptr(), term[i].data_ptr(), imp[i].data_ptr(), None,
                                 B, T, 0.995, 0.90, 1.0, 1.0, adv[i].data_ptr(), None, stream)
        check(rc, L)

    with torch.cuda.stream(st):
        for i in range(S):
            one(i, st.cuda_stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for i in range(S):
                one(i, torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            graph.replay()
        e1.record(st)
        torch.cuda.synchronize()
        t_sets = e0.elapsed_time(e1) / reps / 1e3
        # single-call latency (one set, L2-warm)
        for _ in range(5):
            one(0, st.cuda_stream)
        e0.record(st)
        for _ in range(100):
            one(0, st.cuda_stream)
        e1.record(st)
        torch.cuda.synchronize()
        t_one = e0.elapsed_time(e1) / 100 / 1e3
        # the 64 sets are contiguous and their segments independent, so one launch over S*B segments
        # scans all of them (335 MB > L2): the kernel's own streaming rate without launch gaps
        for _ in range(3):
            check(L.pl_vtrace_f32_dev(rew.data_ptr(), val.data_ptr(), term.data_ptr(), imp.data_ptr(), None, S * B, T,
                                      0.995, 0.90, 1.0, 1.0, adv.data_ptr(), None, st.cuda_stream), L)
        e0.record(st)
        for _ in range(reps):
            check(L.pl_vtrace_f32_dev(rew.data_ptr(), val.data_ptr(), term.data_ptr(), imp.data_ptr(), None, S * B, T,
                                      0.995, 0.90, 1.0, 1.0, adv.data_ptr(), None, st.cuda_stream), L)
        e1.record(st)
        torch.cuda.synchronize()
        t_batched = e0.elapsed_time(e1) / reps / 1e3
    bytes_per_set = 20 * B * T
    gbs_graph = S * bytes_per_set / t_sets / 1e9
    gbs = S * bytes_per_set / t_batched / 1e9
    _, peak_hbm, kind = peaks()
    del graph
    return {"config": "configs[1]: 4096 segments x 64, fp32, gamma .995 lambda .90 rho=c=1",
            "bytes_per_element": 20, "sets": S, "achieved_gbs": gbs_graph, "peak_gbs": peak_hbm,
            "frac": gbs_graph / peak_hbm, "peak_kind": kind,
            "achieved_gbs_how": ("64 launches of the config-sized scan (4096 x 64 each, 5.2 MB) back to back in one "
                                 "CUDA graph over 64 rotating sets (335 MB > L2), consecutive scans overlapping "
                                 "through programmatic dependent launch"),
            "us_per_set": t_sets / S * 1e6, "single_call_us": t_one * 1e6,
            "streaming_gbs": gbs, "streaming_frac": gbs / peak_hbm,
            "streaming_how": "one launch over the 64 contiguous sets (S*B segments): the kernel's streaming rate",
            "elements_per_s": S * B * T / t_sets}


def measure_ns_c3(reps=5):
    """Newton-Schulz (5 quintic steps) on 64 each of 128x128, 512x512 and
    512x2048 bf16 matrices; algorithmic flops 5 (4 m^2 n + 2 m^3) per matrix, 1.035e12 in all."""
    import torch

    import pufferlean_b200 as plb

    L = plb.lib()
    co = np.ascontiguousarray(np.array(QUINTIC, dtype=np.float64))
    dp = C.POINTER(C.c_double)
    groups = [(64, 128, 128), (64, 512, 512), (64, 512, 2048)]
    g = torch.Generator(device="cuda").manual_seed(3)
    Xs = [torch.randn(b, r, c, device="cuda", generator=g).to(torch.bfloat16) for b, r, c in groups]
    flops = sum(b * 5 * (4 * min(r, c) ** 2 * max(r, c) + 2 * min(r, c) ** 3) for b, r, c in groups)

    n = len(groups)
    L.pl_ns_groups_bf16_dev.argtypes = [C.c_size_t, C.POINTER(C.c_void_p)] + [C.POINTER(C.c_size_t)] * 3 + [
        C.c_double, dp, C.c_size_t, C.c_void_p]
    ptrs = (C.c_void_p * n)(*[X.data_ptr() for X in Xs])
    gb, gr, gc = [(C.c_size_t * n)(*[grp[i] for grp in groups]) for i in range(3)]

    def run_grouped():  # the whole config in one call: the two chain batches share one persistent launch
        check(L.pl_ns_groups_bf16_dev(n, ptrs, gb, gr, gc, 1e-7, co.ctypes.data_as(dp), 5, None), L)

    def run_per_shape():  # one pl_ns_batched_bf16_dev call per shape
        for X, (b, r, c) in zip(Xs, groups):
            check(L.pl_ns_batched_bf16_dev(X.data_ptr(), b, r, c, 1e-7, co.ctypes.data_as(dp), 5, None), L)

    def timed(run):
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps / 1e3

    t = timed(run_per_shape)
    t_grouped = timed(run_grouped)
    peak_tf, _, kind = peaks()
    burst = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        burst = json.load(open(p)).get("bf16_tflops")
    tf = flops / t / 1e12
    return {"config": "configs[2]: 64 x {128^2, 512^2, 512x2048}, 5 quintic steps, bf16 in / fp32 acc",
            "flops": flops, "ms": t * 1e3, "achieved_tflops": tf, "peak_tflops": burst or peak_tf,
            "frac": tf / (burst or peak_tf), "peak_kind": kind + " (bf16 burst)",
            "how": "one pl_ns_batched_bf16_dev call per shape (the 512^2 and 512x2048 batches each one persistent "
                   "chain launch, the 128^2 batch the fused one-CTA kernel)",
            "ms_grouped": t_grouped * 1e3,
            "grouped_how": "one pl_ns_groups_bf16_dev call for the three shapes (the two chains share one launch: "
                           "slower here, where each batch fills the GPU alone)"}


def measure_ns_c3_sharded(comm, rank, world, reps=5, chunks=1):
    """configs[2] at N > 1: every group's 64 matrices sharded over the ranks and all-gathered
    (pl_ns_batched_bf16_dev_sharded; each rank orthogonalises its share of a chunk while the previous
    chunk is all-gathered), timed on the device as the max over ranks. Every rank starts from the same
    inputs and ends holding every result. The target time is the slower of the flops over N GPUs at the
    measured burst bf16 rate and the bytes each GPU receives over NVLink at the measured 770 GB/s."""
    import torch
    import torch.distributed as dist

    import pufferlean_b200 as plb

    L = plb.lib()
    co = np.ascontiguousarray(np.array(QUINTIC, dtype=np.float64))
    dp = C.POINTER(C.c_double)
    L.pl_ns_batched_bf16_dev_sharded.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_double, dp,
                                                 C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p]
    L.pl_ns_shard_chunks.argtypes = [C.c_size_t, C.c_size_t, C.c_size_t, C.POINTER(C.c_size_t),
                                     C.POINTER(C.c_size_t)]
    groups = [(64, 128, 128), (64, 512, 512), (64, 512, 2048)]
    g = torch.Generator(device="cuda").manual_seed(3)
    Xs = [torch.randn(b, r, c, device="cuda", generator=g).to(torch.bfloat16) for b, r, c in groups]
    flops = sum(b * 5 * (4 * min(r, c) ** 2 * max(r, c) + 2 * min(r, c) ** 3) for b, r, c in groups)
    recv = 0
    for b, r, c in groups:
        if min(r, c) <= 128 and max(r, c) <= 512:  # whole on every rank (latency-bound fused kernel)
            continue
        cs, used = C.c_size_t(), C.c_size_t()
        check(L.pl_ns_shard_chunks(b, world, chunks, C.byref(cs), C.byref(used)), L)
        recv += used.value * (world - 1) * cs.value * r * c * 2

    def run():
        for X, (b, r, c) in zip(Xs, groups):
            check(L.pl_ns_batched_bf16_dev_sharded(X.data_ptr(), b, r, c, 1e-7, co.ctypes.data_as(dp), 5, comm, chunks,
                                                   None), L)

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps / 1e3], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t = float(t.item())
    peak_tf, _, kind = peaks()
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    burst = json.load(open(p)).get("bf16_tflops") if os.path.exists(p) else None
    burst = burst or peak_tf
    target = max(flops / (world * burst * 1e12), recv / 770e9)
    return {"config": "configs[2] sharded: 64 x {128^2, 512^2, 512x2048} over %d GPUs, %d chunk(s) per group, "
                      "all-gathered (the 128^2 group whole on every rank)" % (world, chunks),
            "n_gpus": world, "flops": flops, "ms": t * 1e3, "achieved_tflops": flops / t / 1e12,
            "allgather_bytes_received_per_gpu": recv, "allgather_gbs_per_gpu": recv / t / 1e9,
            "target_ms": target * 1e3, "frac_of_target": target / t,
            "target_how": "max(flops / (N x measured burst bf16), bytes received per GPU / 770 GB/s peer copy)",
            "peak_kind": kind + " (bf16 burst)"}


WIDE = dict(N=8192, T=64, D=128, H=512, Nmb=65536, epochs=4, lr=0.02)


def measure_wide(args, mode, cpu=True):
    """The wide-action resident update (ffi/puffercuda.cu:1307-1409): one hidden ReLU layer, 8 multi-discrete
    heads of 6 (mode 1, O = 49) or 16 Gaussian dims (mode 2, O = 33); 8192 envs x 64 steps, 4 epochs of
    65,536-row minibatches, value clip and grad-norm clip on. Device leg: the pl_update session with resident
    columns; e2e leg: pl_train_update_wide_resident with host columns (uploads inside the timed region);
    cpu leg: the f64 oracle on one 2,048-row minibatch."""
    import torch

    import pufferlean_b200 as plb

    L = plb.lib()
    dp, vp = C.POINTER(C.c_double), C.c_void_p
    L.pl_update_create.argtypes = [C.c_size_t, C.POINTER(Desc), C.POINTER(vp)]
    L.pl_update_set_head.argtypes = [vp, C.c_int, C.c_size_t, dp]
    L.pl_update_set_columns_dev.argtypes = [vp] * 9
    L.pl_update_run.argtypes = [vp, C.c_double, vp]
    L.pl_update_profile.argtypes = [vp, C.c_int]
    L.pl_update_profile_read.argtypes = [vp, dp, dp, dp]
    L.pl_update_destroy.argtypes = [vp]
    w = WIDE
    NT, D, H, E, Nmb = w["N"] * w["T"], w["D"], w["H"], w["epochs"], w["Nmb"]
    numMB = NT // Nmb
    hs = [6] * 8 if mode == 1 else None
    W = 8 if mode == 1 else 16
    Oo = (sum(hs) if mode == 1 else 2 * W) + 1
    P = H * D + H + Oo * H + Oo
    rng = np.random.default_rng(0x1D + mode)
    fan = np.r_[np.full(H * D + H, D), np.full(Oo * H + Oo, H)]
    pm = np.concatenate([rng.uniform(-1, 1, P) / np.sqrt(fan), np.zeros(P)])
    obs = rng.standard_normal(NT * D).astype(np.float32)
    if mode == 1:
        acts = rng.integers(0, 6, NT * W).astype(np.float64)
        olp = np.full(NT, 8 * np.log(1 / 6)) + 0.05 * rng.standard_normal(NT)
    else:
        acts = rng.standard_normal(NT * W)
        olp = -W * 0.5 * np.log(2 * np.pi * np.e) + 0.05 * rng.standard_normal(NT)
    adv, ret = rng.standard_normal(NT), rng.standard_normal(NT)
    ov = ret + 0.3 * rng.standard_normal(NT)
    perm = plb.shuffle_perm(NT, E, 0x31DE)
    hsa = np.ascontiguousarray(np.array(hs if hs else [0] * W, dtype=np.float64))
    hyp = dict(wd=0.0, mu=0.95, eps=1e-7, vf=0.5, ent=0.01, clip=0.2, vfClip=0.2, maxgn=0.5)
    handle = plb.policy_load(pm, P)
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda()
           for k, v in dict(obs=obs, acts=acts, adv=adv, ret=ret, olp=olp, ov=ov, perm=perm).items()}
    desc = Desc(NT=NT, D=D, H=H, A=Oo - 1, epochs=E, numMB=numMB, arch=Arch(1, 0, None, 0), wd=hyp["wd"],
                mu=hyp["mu"], eps=hyp["eps"], vfCoef=hyp["vf"], entCoef=hyp["ent"], clipEps=hyp["clip"],
                vfClip=hyp["vfClip"], maxGradNorm=hyp["maxgn"], bf16=1, use_old_values=1, rank=0, world=1, comm=None)
    u = vp()
    check(L.pl_update_create(handle, C.byref(desc), C.byref(u)), L)
    check(L.pl_update_set_head(u, mode, W, hsa.ctypes.data_as(dp)), L)
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        check(L.pl_update_set_columns_dev(u, dev["obs"].data_ptr(), dev["acts"].data_ptr(), dev["adv"].data_ptr(),
                                          dev["ret"].data_ptr(), dev["olp"].data_ptr(), dev["ov"].data_ptr(),
                                          dev["perm"].data_ptr(), stream), L)
        check(L.pl_update_run(u, w["lr"], stream), L)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    check(L.pl_update_profile(u, 1), L)
    l0 = L.pl_kernel_launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record()
        for _ in range(args.steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
    launches = L.pl_kernel_launch_count() - l0
    ms = ev0.elapsed_time(ev1) / args.steps
    pms, pfl, pln = (C.c_double * 8)(), (C.c_double * 8)(), (C.c_double * 8)()
    check(L.pl_update_profile_read(u, pms, pfl, pln), L)
    L.pl_update_destroy(u)
    gemm_ms, gemm_fl = sum(pms[i] for i in range(4)), sum(pfl[i] for i in range(4))
    peak_tf, _, kind = peaks()
    achieved = gemm_fl / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
    # e2e: the reference-shaped call with host columns (obs uploaded as f64, as that entry point takes it)
    obs64 = obs.astype(np.float64)
    args_h = (obs64, acts, adv, ret, olp, ov, perm, hs, NT, D, H, Oo, W, mode, E, numMB, w["lr"], hyp["wd"], hyp["mu"],
              hyp["eps"], hyp["vf"], hyp["ent"], hyp["clip"], hyp["vfClip"], hyp["maxgn"], 1)
    plb.cuda_train_update_wide_resident(handle, *args_h)
    reps = max(1, min(args.steps, 3))
    t0 = time.perf_counter()
    for _ in range(reps):
        plb.cuda_train_update_wide_resident(handle, *args_h)
    e2e_s = (time.perf_counter() - t0) / reps
    plb.policy_free(handle)
    out = {"workload": ("wide heads: 8 multi-discrete x 6" if mode == 1 else "wide heads: 16 Gaussian dims") +
           f", MLP {D}->{H}->{Oo} ReLU, {w['N']} envs x {w['T']}, {E} epochs x {numMB} minibatches",
           "unit": "samples/s", "value": NT * E / (ms / 1e3), "ms_per_update": ms,
           "e2e": {"value": NT * E / e2e_s, "unit": "samples/s", "ms_per_update": e2e_s * 1e3,
                   "h2d_bytes_per_step": 8 * (NT * (D + W + 4) + E * NT) + 8 * W},
           "gemm_tflops": achieved, "gemm_frac": achieved / peak_tf if peak_tf else None,
           "gemm_ms_per_update": gemm_ms / args.steps, "peak_kind": kind + " (bf16 sustained)",
           "gpu_launches_per_update": launches / args.steps, "clocks": clk.summary()}
    if cpu:
        from oracle import oracle as O
        n = 2048
        idx = np.arange(n)
        t0 = time.perf_counter()
        O.train_update_wide(pm, obs64[:n * D], acts[:n * W], adv[:n], ret[:n], olp[:n], idx.astype(np.float64), n, D,
                            H, Oo, W, mode, 1, 1, hs=hs, ov=ov[:n], lr=w["lr"], vfClip=0.2, maxGradNorm=0.5)
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": n / dt, "unit": "samples/s", "cores": 1, "kind": "port",
                               "sample": f"one {n}-row minibatch (gradient + clip + Muon), f64 oracle"}
    return out


def measure_lstm(args, cpu=True):
    """The LSTM trainer's per-epoch BPTT gradient (lean_ffi_lstm_ppo_grad_batch_blas*, the reference's 256-env /
    H 64 / T 64 configuration, Puffer/RL/FFITrain.lean:1010-1030) with D 32, A 4: one call = the summed gradient
    over all B*T samples from host columns (the reference-facing call; inputs uploaded and the gradient read
    back inside the timed region), and the same with the inputs reused on the device (epochs > 0). Tiers f32
    (the trainer's production tier) and f64. cpu leg: the f64 oracle on 8 of the 256 sequences."""
    import torch

    import pufferlean_b200 as plb

    B, T, H, D, A = 256, 64, 64, 32, 4
    g = np.random.default_rng(0x15)
    P = plb.lstm_param_count(D, H, A)
    R = B * T
    params = g.uniform(-1, 1, P) / np.sqrt(H)
    cols = [g.standard_normal(R * D), g.integers(0, A, R).astype(float), g.standard_normal(R), g.standard_normal(R),
            g.uniform(-3, -0.3, R), (g.random(R) < 0.01).astype(float), g.uniform(-0.5, 0.5, B * H),
            g.uniform(-0.5, 0.5, B * H)]
    L = plb.lib()
    out = {"workload": f"LSTM BPTT gradient: {B} sequences x {T} steps, D {D} -> LSTM {H} -> {A} + 1", "unit": "samples/s"}
    l0 = L.pl_kernel_launch_count()
    for tier, name in ((1, "f32"), (0, "f64")):
        for reuse in (0, 1):
            plb.cuda_lstm_ppo_grad_batch(params, *cols, B, T, H, D, A, 0.5, 0.01, 0.2, tier=tier)
            L.pl_lstm_reuse_inputs(reuse)
            for _ in range(args.warmup):
                plb.cuda_lstm_ppo_grad_batch(params, *cols, B, T, H, D, A, 0.5, 0.01, 0.2, tier=tier)
            torch.cuda.synchronize()
            reps = max(3, args.steps)
            t0 = time.perf_counter()
            for _ in range(reps):
                plb.cuda_lstm_ppo_grad_batch(params, *cols, B, T, H, D, A, 0.5, 0.01, 0.2, tier=tier)
            dt = (time.perf_counter() - t0) / reps
            L.pl_lstm_reuse_inputs(0)
            key = f"{name}{'_reuse' if reuse else ''}"
            out[key] = {"samples_per_s": R / dt, "ms_per_call": dt * 1e3}
    out["value"] = out["f32"]["samples_per_s"]
    out["gpu_launches_total"] = int(L.pl_kernel_launch_count() - l0)
    if cpu:
        from oracle import oracle as O
        nb = 8
        idx = [t * B + b for t in range(T) for b in range(nb)]
        sub = ([cols[0].reshape(R, D)[idx].ravel()] + [c[idx] for c in cols[1:6]] + [c[:nb * H] for c in cols[6:]])
        t0 = time.perf_counter()
        O.lstm_grad_batch(params, *sub, nb, T, H, D, A)
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": nb * T / dt, "unit": "samples/s", "cores": 1, "kind": "port",
                               "sample": f"{nb} of the {B} sequences, f64 oracle (the reference's scalar BPTT order)"}
    return out


def mingru_init_pm(D, H, L, A, K, seed):
    """[params; mom] in the flattenMG layout, Kaiming-uniform bounds of initMinGRU
    (Puffer/RL/MinGRUTrain.lean:311-344: sqrt(2)/sqrt(D) encoder, 1/sqrt(H) elsewhere, biases zero),
    drawn with numpy from `seed` (random-init weights of the named architecture)."""
    g = np.random.default_rng(seed)
    parts = [g.uniform(-1, 1, H * D) * np.sqrt(2.0 / D), np.zeros(H)]
    parts += [g.uniform(-1, 1, K * H * H) / np.sqrt(H) for _ in range(L)]
    parts += [g.uniform(-1, 1, A * H) / np.sqrt(H), np.zeros(A), g.uniform(-1, 1, H) / np.sqrt(H), np.zeros(1)]
    p = np.concatenate(parts)
    return p.size, np.concatenate([p, np.zeros(p.size)])


MINGRU_C4 = dict(N=8192, T=64, D=118, H=512, L=1, A=4, mb_segs=512, num_mb=64, lr=0.02)


def measure_mingru_c4(args, K=2, enc_act=1, steps=None, warmup=None, cpu=False, comm=None, rank=0, world=1):
    """the Breakout-shaped recurrent update, 8192 envs x 64, obs 118 ~U(0,1), 4 actions,
    rewards U(-1,1), dones Bernoulli(.005); encoder 118->512 (+GELU), MinGRU hidden 512 with gate + candidate
    512->1024 (K = 2; K = 3 adds the reference's highway projection), heads 512->4 and 512->1; minibatches of
    32768 rows (512 segments x 64) x 64 per update (16 x 4 epochs), each: device V-trace over all 8192 segments,
    prioritised sampling, BPTT gradient, value/ratio iterate, clip, Muon. samples/s = N*T / update time.
    With world > 1 every rank holds its own 8192-env rollout (weak scaling) and the ranks all-reduce the
    advantage statistics and the gradient of every minibatch (pl_mg_set_comm); the time is the max over
    ranks and the value world * N*T / time."""
    import torch

    import pufferlean_b200 as plb

    c = MINGRU_C4
    N, T, D, H, L_, A = c["N"], c["T"], c["D"], c["H"], c["L"], c["A"]
    NT = N * T
    L = plb.lib()
    gen = torch.Generator(device="cuda").manual_seed(4 + 1000 * rank)
    obs = torch.rand(NT * D, device="cuda", generator=gen)
    rew = torch.rand(NT, device="cuda", generator=gen, dtype=torch.float64) * 2 - 1
    term = (torch.rand(NT, device="cuda", generator=gen) < 0.005).double()
    act = torch.randint(0, A, (NT,), device="cuda", generator=gen).double()
    logp = torch.full((NT,), float(np.log(1.0 / A)), device="cuda", dtype=torch.float64) + \
        0.05 * torch.randn(NT, device="cuda", generator=gen, dtype=torch.float64)
    val = torch.randn(NT, device="cuda", generator=gen, dtype=torch.float64)
    boot = torch.randn(N, device="cuda", generator=gen, dtype=torch.float64)
    P, pm = mingru_init_pm(D, H, L_, A, K, 44)
    handle = plb.policy_load(pm, P)
    net = plb.mg_net(D, H, L_, A, K, enc_act)
    co = np.ascontiguousarray(np.array(QUINTIC, dtype=np.float64))
    hy = plb.MgHyper(gamma=0.995, lam=0.90, rhoClip=1.0, cClip=1.0, prioAlpha=0.8, annealBeta=0.2, wd=0.0, mu=0.95,
                     eps=1e-12, vfCoef=0.5, entCoef=0.01, clipEps=0.2, vfClip=0.2, maxGradNorm=1.5,
                     ns_coeffs=co.ctypes.data_as(C.POINTER(C.c_double)), ns_iters=5, bf16=1)
    s = plb.MgSession(N, T)
    if world > 1:
        s.set_comm(comm, rank, world)
    st = torch.cuda.current_stream().cuda_stream
    check(L.pl_mg_set_obs_dev(s.h, obs.data_ptr(), D), L)
    rng = [0x5EED]

    def step():
        check(L.pl_mg_set_columns_dev(s.h, rew.data_ptr(), term.data_ptr(), act.data_ptr(), logp.data_ptr(),
                                      val.data_ptr(), boot.data_ptr(), st), L)
        r = C.c_uint64(rng[0])
        check(L.pl_mg_update(s.h, C.byref(net), handle, C.byref(hy), c["num_mb"], c["mb_segs"], C.byref(r), c["lr"],
                             st), L)
        rng[0] = r.value

    steps = steps or max(2, min(args.steps, 5))
    warmup = warmup or max(3, args.warmup)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    l0 = L.pl_kernel_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    launches = (L.pl_kernel_launch_count() - l0) / steps
    pm_out = plb.policy_download(handle, P)
    plb.policy_free(handle)
    s.close()
    R = c["mb_segs"] * T
    Op = A + 1
    # algorithmic GEMM flops per minibatch: forward enc/layer/heads, backward dW of all + dX of layer/heads
    fwd = 2 * R * (D * H + L_ * H * K * H + H * Op)
    bwd = 2 * R * (D * H + L_ * 2 * H * K * H + 2 * H * Op)
    flops = (fwd + bwd) * c["num_mb"]
    m_ns = [(H, D)] + [(K * H, H)] * L_ + [(A, H), (1, H)]
    ns_fl = sum(5 * (4 * min(r_, c_) ** 2 * max(r_, c_) + 2 * min(r_, c_) ** 3) for r_, c_ in m_ns) * c["num_mb"]
    out_cpu = None
    if cpu:
        from oracle import cpu_port

        per_update, det = cpu_port.mingru_timed_sample(D, H, L_, A, K, enc_act, T, c["mb_segs"], c["num_mb"], QUINTIC)
        out_cpu = {"value": NT / per_update, "unit": "samples/s", "cores": det["threads"],
                   "kind": "reference" if det["grad_source"] == "reference C" else "port",
                   "sample": (f"BPTT gradient of {det['nseq']} sequences x {T} steps, one per host thread "
                              f"({det['grad_source']}, ffi/pufferffi.c:763-876; {det['t_grad']:.2f} s) + one Muon "
                              f"step of every matrix on numpy BLAS ({det['t_muon']:.2f} s), scaled to "
                              f"{c['num_mb']} minibatches of {c['mb_segs']} sequences")}
    return {"cpu_baseline": out_cpu,
            "config": "configs[3]: Breakout-shaped MinGRU update, 8192 envs x 64, obs 118, H 512, "
                      f"{'gate+candidate 512->1024 (K=2)' if K == 2 else 'hid|gate|proj 512->1536 (K=3, reference)'}"
                      f"{', GELU encoder' if enc_act else ''}, 4 actions, 64 minibatches of 512 segments x 64",
            "K": K, "enc_act": "gelu" if enc_act else "none", "params": P,
            "n_gpus": world, "scaling": "weak",
            "value": world * NT / (ms / 1e3), "unit": "samples/s", "ms_per_update": ms,
            "gpu_launches_per_update": launches,
            "gemm_tflops_over_update": flops / (ms / 1e3) / 1e12, "ns_flops_per_update": ns_fl,
            "finite": bool(np.isfinite(pm_out).all()), "data": "synthetic (seeded torch generator 4)"}


def _mlp_loss(pm, obs, acts, adv, ret, olp, D, H, A, vf=0.5, ent=0.01, clip=0.2):
    """PPO loss of the one-hidden-layer ReLU policy (the reference's MLP) on the whole buffer, f64:
    -mean(min(adv r, adv clip(r))) + vf 0.5 mean((v - ret)^2) - ent mean(entropy)."""
    W1 = pm[:H * D].reshape(H, D)
    b1 = pm[H * D:H * D + H]
    O = A + 1
    W2 = pm[H * D + H:H * D + H + O * H].reshape(O, H)
    b2 = pm[H * D + H + O * H:H * D + H + O * H + O]
    h = np.maximum(obs @ W1.T + b1, 0.0)
    out = h @ W2.T + b2
    lg, v = out[:, :A], out[:, A]
    m = lg.max(axis=1, keepdims=True)
    lse = m[:, 0] + np.log(np.exp(lg - m).sum(axis=1))
    p = np.exp(lg - lse[:, None])
    logp = lg[np.arange(len(acts)), acts.astype(int)] - lse
    r = np.exp(logp - olp)
    pg = -np.mean(np.minimum(adv * r, adv * np.clip(r, 1 - clip, 1 + clip)))
    entropy = np.mean(lse - (p * lg).sum(axis=1))
    return float(pg + vf * 0.5 * np.mean((v - ret) ** 2) - ent * entropy)


def measure_drift(updates=100):
    """Loss-curve drift over `updates` consecutive updates: the reference's MLP (configs[0] shapes with
    its own net: 4 -> 128 ReLU -> 2 + 1, Kaiming init, its Newton-Schulz table) trained on one fixed
    seeded 64 x 64 buffer by this library (bf16 and fp32 tiers, the resident update through the C ABI)
    and by the oracle (f64 restatement of the reference CPU update), identical inputs and shuffles.
    Reports the PPO loss of both parameter trajectories on the whole buffer after every update."""
    import pufferlean_b200 as plb
    from oracle import oracle as O

    N, T, D, H, A, E, MB = 64, 64, 4, 128, 2, 4, 4
    NT = N * T
    g = np.random.default_rng(11)
    obs = g.standard_normal(NT * D)
    acts = g.integers(0, A, NT).astype(np.float64)
    rew = (g.random(NT) < 0.5).astype(np.float64)
    term = (g.random(NT) < 0.01).astype(np.float64)
    params, _ = O.init_mlp(D, H, A + 1, 0xD21F7)
    P = params.size
    pm0 = np.concatenate([params, np.zeros(P)])
    _, olp, val = O.mlp_ppo_grad(params, obs, acts, np.zeros(NT), np.zeros(NT), np.zeros(NT), NT, D, H, A)
    ga = O.gae_soa(val, rew, term, N, T, 0.995, 0.90)
    adv, ret = ga[:NT], ga[NT:]
    hyper = dict(lr=0.02, wd=0.0, mu=0.95, eps=1e-7, vf=0.5, ent=0.01, clip=0.2, vfClip=0.2, maxGradNorm=1.5)
    ob2 = obs.reshape(NT, D)

    def loss(pm):
        return _mlp_loss(pm[:P], ob2, acts, adv, ret, olp, D, H, A)

    cpu = pm0.copy()
    # control: the same f64 oracle from weights perturbed by 1e-12 (relative), to separate the
    # divergence the training dynamics amplify from any implementation difference
    ctl = pm0.copy()
    ctl[:P] *= 1.0 + 1e-12 * np.random.default_rng(12).standard_normal(P)
    curves = {"oracle_f64": [loss(cpu)], "oracle_perturbed_1e-12": [loss(ctl)]}
    handles = {"bf16": plb.policy_load(pm0, P), "fp32": plb.policy_load(pm0, P)}
    for k in handles:
        curves[k] = [curves["oracle_f64"][0]]
    t0 = time.time()
    for u in range(updates):
        perm = plb.shuffle_perm(NT, E, 1000 + u)
        cpu = O.train_update(cpu, obs, acts, adv, ret, olp, perm, NT, D, H, A, E, MB, hyper["lr"], hyper["wd"],
                             hyper["mu"], hyper["eps"], hyper["vf"], hyper["ent"], hyper["clip"], ov=val,
                             vfClip=hyper["vfClip"], maxGradNorm=hyper["maxGradNorm"])
        curves["oracle_f64"].append(loss(cpu))
        ctl = O.train_update(ctl, obs, acts, adv, ret, olp, perm, NT, D, H, A, E, MB, hyper["lr"], hyper["wd"],
                             hyper["mu"], hyper["eps"], hyper["vf"], hyper["ent"], hyper["clip"], ov=val,
                             vfClip=hyper["vfClip"], maxGradNorm=hyper["maxGradNorm"])
        curves["oracle_perturbed_1e-12"].append(loss(ctl))
        for k, h in handles.items():
            plb.cuda_train_update_resident(h, obs, acts, adv, ret, olp, val, perm, NT, D, H, A, E, MB, hyper["lr"],
                                           hyper["wd"], hyper["mu"], hyper["eps"], hyper["vf"], hyper["ent"],
                                           hyper["clip"], hyper["vfClip"], hyper["maxGradNorm"], 1 if k == "bf16" else 0)
            curves[k].append(loss(plb.policy_download(h, P)))
    finals = {k: plb.policy_download(h, P)[:P] for k, h in handles.items()}
    for h in handles.values():
        plb.policy_free(h)
    ref = np.array(curves["oracle_f64"])
    res = {"config": "configs[0] shapes, the reference's MLP (4 -> 128 ReLU -> 2+1), one fixed seeded 64 x 64 buffer, "
                     f"{E} epochs x {MB} minibatches per update, {updates} updates",
           "loss_first": float(ref[0]), "loss_last_oracle": float(ref[-1]), "seconds": time.time() - t0}
    scale = float(np.max(np.abs(ref - ref[0]))) or 1.0
    res["oracle_mean_loss_updates_51_100"] = float(np.mean(ref[51:]))
    for k in list(handles) + ["oracle_perturbed_1e-12"]:
        c = np.array(curves[k])
        d = np.abs(c - ref)
        res[k] = {"loss_last": float(c[-1]), "max_abs_drift": float(d.max()),
                  "max_drift_rel_to_loss_change": float(d.max() / scale),
                  "drift_at": {str(u): float(d[u]) for u in sorted({1, 5, 10, 50, updates}) if u <= updates},
                  "mean_loss_updates_51_100": float(np.mean(c[51:])) if updates > 51 else None,
                  "param_rel_diff": float(np.linalg.norm((finals[k] if k in finals else ctl[:P]) - cpu[:P]) /
                                          np.linalg.norm(cpu[:P] - pm0[:P]))}
    res["curve_oracle_every10"] = [float(x) for x in ref[::10]]
    res["curve_bf16_every10"] = [float(x) for x in np.array(curves["bf16"])[::10]]
    return res


def cudart_memcpy_d2h(dst, handle):
    """8-byte read-back of params[0] from the resident policy (the reference's divergence guard)."""
    import pufferlean_b200 as plb

    L = plb.lib()
    L.pl_policy_download.argtypes = [C.c_size_t, C.c_size_t, C.POINTER(C.c_double)]
    buf = np.zeros(2)
    # a 1-parameter download reads [params[0]; params[1]]: the first 16 bytes of the handle
    check(L.pl_policy_download(handle, 1, buf.ctypes.data_as(C.POINTER(C.c_double))), L)
    dst[0] = buf[0]


def cpu_baseline(wl, steps=1):
    from oracle import cpu_port

    try:
        from threadpoolctl import threadpool_info

        threads = max([x.get("num_threads", 1) for x in threadpool_info()] or [os.cpu_count()])
    except Exception:
        threads = os.cpu_count()
    vals, det = [], None
    for s in range(steps):
        per_update, det = cpu_port.timed_update_sample(wl["D"], wl["H"], wl["A"], wl["L"], wl["act"], wl["Nmb"],
                                                       wl["epochs"], wl["N"] * wl["T"] // wl["Nmb"],
                                                       QUINTIC, rows=4096, seed=s)
        vals.append(wl["N"] * wl["T"] / per_update)
    return {"value": float(np.mean(vals)), "unit": "samples/s", "cores": int(threads), "kind": "port",
            "sample": ("numpy f64 restatement of the reference's pufferblas CPU update (oracle/cpu_port.py): one "
                       f"minibatch gradient on {det['rows']} rows ({det['t_rows']:.2f} s) + one whole-network Muon "
                       f"step ({det['t_muon']:.2f} s), scaled to {wl['epochs']} epochs x "
                       f"{wl['N'] * wl['T'] // wl['Nmb']} minibatches of {wl['Nmb']} rows")}


def reference_c1(wl, steps, warmup):
    """configs[0] through the reference's own compiled C (oracle/_ref/libref_cpu.so, composed as its CPU
    trainer calls it: oracle/ref_update.py) on every host core: whole updates, same shapes, init and
    hyperparameters as this library's C1 line."""
    from oracle import ref_update as R

    N, T, D, H, A = wl["N"], wl["T"], wl["D"], wl["H"], wl["A"]
    NT, E = N * T, wl["epochs"]
    g = np.random.default_rng(7)
    _, pm = xavier_pm(D, H, A, 1, 42)
    cols = (g.standard_normal(NT * D), g.integers(0, A, NT).astype(float),
            np.log(1.0 / A) + 0.05 * g.standard_normal(NT), g.standard_normal(NT),
            (g.random(NT) < 0.5).astype(float), (g.random(NT) < wl["done"]).astype(float))
    dt, pm, threads = R.timed_updates(pm, cols, N, T, D, H, A, E, NT // wl["Nmb"], steps, warmup, lr=wl["lr"],
                                      eps=1e-12, max_grad_norm=wl["maxgn"])
    return {"value": NT / dt, "unit": "samples/s", "cores": int(threads), "kind": "reference",
            "sample": (f"{steps} whole updates ({dt:.3f} s each) through the reference's compiled C: lean_ffi_gae_soa, "
                       "lean_ffi_shuffle_perm, per minibatch lean_ffi_gather_minibatch, normalizeAdv (restatement), "
                       "lean_ffi_mlp_ppo_grad_batch_blas, the mean-gradient clip, lean_ffi_muon_step_mlp; BLAS "
                       f"threads {threads} (lean_ffi_blas_set_threads)"),
            "finite": bool(np.isfinite(pm).all())}


def measure_c1(args):
    """configs[0] on this library (device-resident update and the reference-facing call from host
    columns) beside the reference's own compiled C on the host cores."""
    import pufferlean_b200 as plb

    wl = WORKLOADS["c1"]
    a = argparse.Namespace(**vars(args))
    a.steps, a.warmup = 20, 3
    out, state = run_ours(a, wl, 0, 1, 0)
    e2e = run_e2e(a, wl, state, 0, 1, 0)
    plb.policy_free(state["handle"])
    res = {"config": wl["name"], "dtype": "f32 (tight tier: fp32 GEMMs, f64 Muon)", "value": out["value"],
           "ms_per_step": out["ms_per_step"], "gpu_launches_per_update": out["gpu_launches"] / a.steps,
           "l2": out["config"]["l2"], "e2e": e2e}
    if not args.no_cpu and os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libref_cpu.so")):
        ref = reference_c1(wl, 3, 1)
        res["reference_c"] = ref
        res["device_over_reference"] = out["value"] / ref["value"]
        res["e2e_over_reference"] = e2e["value"] / ref["value"]
    return res


def _all_cores_blas():
    """Every host core for numpy's BLAS, whatever OMP_NUM_THREADS the launcher set."""
    try:
        from threadpoolctl import threadpool_limits

        from oracle.ref_update import host_cores

        return threadpool_limits(limits=host_cores(), user_api="blas")
    except Exception:
        import contextlib

        return contextlib.nullcontext()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c5")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="N > 1: weak = every rank its own rollout of the workload's size; strong = one rollout of "
                         "that size, each minibatch split over the ranks (value = that rollout's samples / time)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the configs[1] / configs[2] kernel measurements")
    ap.add_argument("--drift", type=int, default=0, metavar="U",
                    help="print the loss-curve drift of U consecutive updates against the f64 oracle and exit")
    ap.add_argument("--only", choices=["c2", "c3", "c4", "c4r", "wide1", "wide2", "lstm"],
                    help="print only the configs[1] (c2), configs[2] (c3) or configs[3] (c4: K=2 + GELU encoder; "
                         "c4r: the reference's K=3 linear-encoder net) measurement, or the wide-head update "
                         "(wide1 multi-discrete, wide2 Gaussian), or the LSTM BPTT gradient (lstm)")
    args = ap.parse_args()
    if args.drift:
        print(json.dumps(measure_drift(args.drift)), flush=True)
        return 0
    if args.only:
        if args.only == "c4":
            res = measure_mingru_c4(args, cpu=not args.no_cpu)
        elif args.only == "c4r":
            res = measure_mingru_c4(args, K=3, enc_act=0, cpu=not args.no_cpu)
        elif args.only in ("wide1", "wide2"):
            res = measure_wide(args, int(args.only[-1]), cpu=not args.no_cpu)
        elif args.only == "lstm":
            res = measure_lstm(args, cpu=not args.no_cpu)
        else:
            res = measure_vtrace_c2() if args.only == "c2" else measure_ns_c3()
        print(json.dumps(res), flush=True)
        return 0
    wl = WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        if args.workload == "c1":
            base = reference_c1(wl, max(1, args.steps), min(args.warmup, 1))
        else:
            with _all_cores_blas():
                base = cpu_baseline(wl, steps=max(1, min(args.steps, 2)))
        line = {"metric": METRIC, "value": base["value"], "unit": "samples/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f64", "data": "synthetic (seeded)", "impl": "reference",
                "config": {"workload": wl["name"], "parallelism": "host cores (%d)" % base["cores"]},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        import datetime

        import torch

        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    early = {}
    if world == 1 and not args.no_extra:
        # the configs[1] / configs[2] kernel measurements first, on a GPU not yet held at its power cap by
        # seconds of the update (their peaks are the burst figures)
        early["c2_vtrace"] = measure_vtrace_c2()
        early["c3_newton_schulz"] = measure_ns_c3()
    out, state = run_ours(args, wl, rank, world, local_rank)
    if not args.no_e2e:
        out["e2e"] = run_e2e(args, wl, state, rank, world, local_rank)
    import pufferlean_b200 as plb

    plb.policy_free(state["handle"])
    if world > 1 and args.scaling == "weak":
        # the same workload as ONE rollout with each minibatch split over the ranks (strong scaling),
        # device-resident, on the same communicator
        a2 = argparse.Namespace(**vars(args))
        a2.scaling = "strong"
        s_out, s_state = run_ours(a2, wl, rank, world, local_rank, comm=state["comm"])
        plb.policy_free(s_state["handle"])
        if rank == 0:
            out["strong_scaling"] = {k: s_out[k] for k in ("value", "unit", "ms_per_step", "scaling", "dp_allreduce",
                                                           "gpu_launches")}
            out["strong_scaling"]["config"] = s_out["config"]
            out["strong_scaling"]["profile"] = s_out["profile"]
    if world > 1 and not args.no_extra:
        # configs[3] and configs[2] on every rank (their multi-GPU forms), before the communicator goes away
        c4 = measure_mingru_c4(args, comm=state["comm"], rank=rank, world=world)
        c3s = measure_ns_c3_sharded(state["comm"], rank, world)
        if rank == 0:
            out["c4_mingru"] = c4
            out["c3_newton_schulz_sharded"] = c3s
    if state.get("comm"):
        plb.lib().pl_comm_destroy.argtypes = [C.c_void_p]
        plb.lib().pl_comm_destroy(state["comm"])
    if rank == 0 and not args.no_extra:
        out["c2_vtrace"] = early.get("c2_vtrace") or measure_vtrace_c2()
        out["c3_newton_schulz"] = early.get("c3_newton_schulz") or measure_ns_c3()
        if world == 1:
            out["c4_mingru"] = measure_mingru_c4(args, cpu=not args.no_cpu)
            if args.workload != "c1":
                out["c1_cartpole"] = measure_c1(args)
    if rank == 0:
        if not args.no_cpu and world == 1:
            if args.workload == "c1":
                out["cpu_baseline"] = reference_c1(wl, 3, 1)
            else:
                with _all_cores_blas():
                    out["cpu_baseline"] = cpu_baseline(wl)
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch

        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
