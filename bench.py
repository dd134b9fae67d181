"""Benchmark of the fused RMSNorm + RoPE path, forward + backward.

One step = one training-style pass of the path over one batch: the hidden-state
RMSNorm forward (``bloth_b200.rms_norm``), the q/k per-head RMSNorm + RoPE
forward (``bloth_b200.fused_qk_norm_rope``, cos/sin from positions
in-register), then the backward of both for given output gradients (dx,
dweight, dq, dk, dwq, dwk) via ``torch.autograd.grad``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl b200|reference|reference-triton]
                    [--scaling weak|strong] [--shard-of N]

N > 1 is launched with torch.distributed.run, one rank per GPU; every rank
processes its own contiguous shard of batch rows (no collective on the data
path); the step time is the max over ranks. Prints one JSON line on rank 0.

Scaling. The Llama-3-8B and the Qwen3-8B packed workloads are defined as one
batch whose token rows are sharded over the GPUs, so they default to strong
scaling: at N GPUs each rank takes batch/N rows (Llama-3-8B: 32768 tokens on
one GPU, 4096 per GPU on eight). The other workloads default to weak scaling
(the full batch on every rank). ``--shard-of N`` runs, on one GPU, the shard
that rank 0 of an N-rank strong-scaling job processes.

Checks. After the timed region every rank reads the library's device fault
word and re-runs one step whose results are checked: sampled tokens of the
rank's shard against the CPU oracle, and the weight gradients summed over the
ranks (one all-reduce, outside the timed region) against the float64 oracle
over the whole batch and, at N > 1, against the same kernels run over the
whole batch on one GPU. The line carries ``fault`` and ``parity_ok``.

``--impl reference`` times the reference's CPU path instead: the oracle's
PyTorch restatement in float32 on all host cores, on a fixed sample of the
same workload per step (the reference has no CPU implementation of its own).
``--impl reference-triton`` times the reference's own Triton kernels from the
package installed under baseline/_ref (one GPU).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "fused RMSNorm+RoPE fwd+bwd tokens/s and HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"

# DRAM bytes (read + write) of one step's launches of each C-ABI call at the
# Llama-3-8B shape, from the ncu captures summarised in profiles/ (cold L2; a
# backward's dweight reduce launch moves under 1 MB and is not included).
PROFILED_TRAFFIC = {
    ("llama3-8b", "bloth_qk_norm_rope_fwd"): 335_875_072 + 285_793_024,
    ("llama3-8b", "bloth_qk_norm_rope_bwd"): 676_634_368 + 300_522_752,
    ("llama3-8b", "bloth_rmsnorm_fwd"): 268_538_368 + 216_425_984,
    ("llama3-8b", "bloth_rmsnorm_bwd"): 537_050_112 + 239_020_544,
    # reference-contract rows: the q and the k launch of the call together
    ("llama3-8b-rows", "bloth_norm_rope_fwd"): 536_897_280 + 224_008_704 + 134_242_304 + 20_562_944,
    ("llama3-8b-rows", "bloth_norm_rope_bwd"): 809_656_576 + 244_946_432 + 202_408_960 + 42_970_112,
}
NOMINAL_HBM_GBS = 8000.0

# name -> (batch, seq, hidden (0 = none), heads_q, heads_kv, head_dim, theta, eps, packed)
WORKLOADS = {
    "llama3-8b": (8, 4096, 4096, 32, 8, 128, 5e5, 1e-5, False),
    "llama3.2-1b": (4, 2048, 2048, 32, 8, 64, 5e5, 1e-5, False),
    "qwen3-8b-packed": (16, 8192, 0, 32, 8, 128, 1e6, 1e-6, True),
    # as llama3-8b, with the hidden RMSNorm preceded by the residual add
    # (fused_add_rms_norm: z = x + r, y = RMSNorm(z); z's gradient from the
    # residual stream joins in the backward)
    "llama3-8b-residual": (8, 4096, 4096, 32, 8, 128, 5e5, 1e-5, False),
    # as llama3-8b, through the reference's own entry points: rms_norm, and
    # fused_norm_rope on q and k as rows of head_dim with per-row cos/sin
    # tables [rows, head_dim/2] (bf16, expanded across heads, as the
    # reference's contract requires)
    "llama3-8b-rows": (8, 4096, 4096, 32, 8, 128, 5e5, 1e-5, False),
}
RESIDUAL = {"llama3-8b-residual"}
ROWS = {"llama3-8b-rows"}
# workloads defined as one batch whose token rows are sharded over the GPUs
SHARDED = {"llama3-8b", "qwen3-8b-packed"}

# tokens per step of the CPU timings (the reference arm and the GPU arm's
# cpu_baseline leg time the same sample), and their minimum duration
CPU_SAMPLE_TOKENS = 512
CPU_MIN_SECONDS = 12.0


def describe(name: str) -> str:
    B, S, Hd, Hq, Hk, D, theta, eps, packed = WORKLOADS[name]
    parts = []
    if Hd:
        parts.append(f"hidden [{B},{S},{Hd}] " +
                     ("residual add + RMSNorm" if name in RESIDUAL else "RMSNorm"))
    if name in ROWS:
        parts.append(f"q [{B},{S},{Hq},{D}] + k [{B},{S},{Hk},{D}] as rows of {D} through "
                     f"fused_norm_rope with per-row bf16 cos/sin tables [rows, {D // 2}]")
    else:
        parts.append(f"q [{B},{S},{Hq},{D}] + k [{B},{S},{Hk},{D}] norm+RoPE")
    extra = ", packed documents (lengths U[64,2048])" if packed else ""
    return f"{name}: " + " + ".join(parts) + f", bf16, theta {theta:g}, eps {eps:g}{extra}"


def step_bytes(tokens: int, name: str, elem: int = 2) -> dict:
    """Algorithmic HBM bytes of one fwd+bwd step over `tokens` tokens.

    Per normalised row of width W: forward reads x and writes y (2*W*s) and
    writes rstd (4 B); backward reads dy and x and writes dx (3*W*s) and reads
    rstd (4 B). Positions are int64: 8 B per token per pass. Weights and
    dweight (a few KB) are not counted. Through the per-row table contract
    each head row also reads its cos and sin rows (2 * D/2 * s) in each pass,
    and there are no positions.
    """
    _, _, Hd, Hq, Hk, D, _, _, _ = WORKLOADS[name]
    rows = Hq + Hk
    if name in RESIDUAL:
        # forward reads x, r and writes z, y; backward reads dy, z, dz_out and
        # writes dz
        hid = {"add_fwd": tokens * (4 * Hd * elem + 4), "add_bwd": tokens * (4 * Hd * elem + 4)}
    else:
        hid = {"rms_fwd": tokens * (2 * Hd * elem + 4) if Hd else 0,
               "rms_bwd": tokens * (3 * Hd * elem + 4) if Hd else 0}
    if name in ROWS:
        tab = 2 * (D // 2) * elem
        out = {**hid,
               "nr_fwd": tokens * rows * (2 * D * elem + 4 + tab),
               "nr_bwd": tokens * rows * (3 * D * elem + 4 + tab)}
    else:
        out = {
            **hid,
            "qk_fwd": tokens * (rows * (2 * D * elem + 4) + 8),
            "qk_bwd": tokens * (rows * (3 * D * elem + 4) + 8),
        }
    out["total"] = sum(out.values())
    return out


# ------------------------------------------------------------- ranks
def default_scaling(name: str) -> str:
    """Strong scaling (the batch's rows split over the ranks) for the
    workloads defined as one sharded batch, weak scaling otherwise."""
    return "strong" if name in SHARDED else "weak"


def local_batch(batch: int, world: int, scaling: str) -> int:
    """Batch rows (sequences) one rank processes: the full batch per rank
    under weak scaling, an equal share of it under strong scaling."""
    if scaling == "weak":
        return batch
    if batch % world:
        raise ValueError(f"strong scaling needs batch {batch} divisible by {world} ranks")
    return batch // world


def shard_rows(batch: int, world: int, rank: int, scaling: str) -> range:
    """Global batch-row indices of `rank`'s shard: a contiguous block of
    batch/world rows under strong scaling; under weak scaling every rank
    takes a full batch of its own (rows rank*batch ...), so that the inputs of
    different ranks differ."""
    b = local_batch(batch, world, scaling)
    return range(rank * b, (rank + 1) * b)


def max_over_ranks(value: float, dist, device) -> float:
    """Largest `value` over all ranks (the job finishes with its slowest rank);
    `value` itself when not distributed."""
    if dist is None:
        return value
    import torch as _t
    t = _t.tensor([value], device=device, dtype=_t.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------- inputs
def _row_seed(seed: int, row: int) -> int:
    return seed * 100003 + 7919 * (row + 1)


def make_inputs(name: str, rows, dev, seed: int = 1234):
    """Seeded synthetic inputs on `dev` for the batch rows `rows` (a range of
    global batch-row indices, or a count meaning range(count)).

    Every batch row (sequence) is drawn from its own generator seeded by
    (seed, row), so a rank's shard holds exactly the rows of the whole batch
    it covers, wherever it is generated. Weights depend on `seed` only (they
    are replicated on every rank)."""
    if isinstance(rows, int):
        rows = range(rows)
    B, S, Hd, Hq, Hk, D, theta, eps, packed = WORKLOADS[name]
    bf = torch.bfloat16
    b = len(rows)
    wg = torch.Generator(device=dev).manual_seed(seed)

    def weight(n):
        return (1 + 0.1 * torch.randn(n, generator=wg, device=dev)).to(bf)

    shapes = {}
    if Hd:
        shapes["x"] = (S, Hd)
        shapes["gy"] = (S, Hd)
        if name in RESIDUAL:
            shapes["r"] = (S, Hd)
            shapes["gz"] = (S, Hd)
    shapes.update(q=(S, Hq, D), k=(S, Hk, D), gq=(S, Hq, D), gk=(S, Hk, D))
    inp = {key: torch.empty((b, *shp), dtype=bf, device=dev) for key, shp in shapes.items()}
    for i, r in enumerate(rows):
        g = torch.Generator(device=dev).manual_seed(_row_seed(seed, r))
        for key, shp in shapes.items():
            inp[key][i].copy_(torch.randn(*shp, generator=g, device=dev, dtype=torch.float32))
    if Hd:
        inp["w"] = weight(Hd)
    inp["wq"] = weight(D)
    inp["wk"] = weight(D)
    if packed:
        from oracle.reference_path import packed_position_ids  # seeded document layout
        pos = torch.cat([packed_position_ids(1, S, 64, 2048,
                                             torch.Generator().manual_seed(_row_seed(seed, r)))
                         for r in rows]) if b else torch.empty(0, S, dtype=torch.int64)
        inp["pos"] = pos.to(dev)
    else:
        inp["pos"] = torch.arange(S, device=dev, dtype=torch.int64).expand(b, S).contiguous()
    half = D // 2
    inp["inv_freq"] = (1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))).to(dev)
    inp["eps"] = eps
    if name in ROWS:
        # per-row tables of the reference's contract: the angle of every
        # (token, pair) evaluated in fp32, stored in bf16, expanded per head
        ang = inp["pos"].to(torch.float32)[..., None] * inp["inv_freq"]
        for key, H in (("q", Hq), ("k", Hk)):
            for fn in ("cos", "sin"):
                t = getattr(torch, fn)(ang).to(bf)[:, :, None, :].expand(b, S, H, half)
                inp[f"{fn}_{key}"] = t.reshape(-1, half).contiguous()
    return inp


def merge_summaries(sums: list) -> dict:
    """Per-call breakdown over several instrumented steps: the call's
    launches in one step, and the median over the steps of its time in a
    step."""
    out = {}
    for name in sums[0]:
        per_step = sorted(s[name]["total_ms"] for s in sums if name in s)
        med = per_step[len(per_step) // 2]
        n = sums[0][name]["launches"]
        out[name] = {"launches": n, "total_ms": med, "mean_ms": med / n}
    return out


def run_step(inp, bloth):
    """One fwd+bwd pass through the public API; returns (outputs, gradients)
    as dicts keyed by name."""
    leaves, outs, grads = {}, {}, []
    if "r" in inp:
        x = inp["x"].requires_grad_(True)
        r = inp["r"].requires_grad_(True)
        w = inp["w"].requires_grad_(True)
        outs["y"], outs["z"] = bloth.fused_add_rms_norm(x, r, w, inp["eps"])
        grads += [inp["gy"], inp["gz"]]
        leaves.update(dx=x, dr=r, dw=w)
    elif "x" in inp:
        x = inp["x"].requires_grad_(True)
        w = inp["w"].requires_grad_(True)
        outs["y"] = bloth.rms_norm(x, w, inp["eps"])
        grads.append(inp["gy"])
        leaves.update(dx=x, dw=w)
    q = inp["q"].requires_grad_(True)
    k = inp["k"].requires_grad_(True)
    wq = inp["wq"].requires_grad_(True)
    wk = inp["wk"].requires_grad_(True)
    if "cos_q" in inp:  # the reference's per-row table contract, one call per tensor
        qo = bloth.kernels.fused_norm_rope(q, wq, inp["cos_q"], inp["sin_q"], inp["eps"])
        ko = bloth.kernels.fused_norm_rope(k, wk, inp["cos_k"], inp["sin_k"], inp["eps"])
    else:
        qo, ko = bloth.fused_qk_norm_rope(q, k, wq, wk, inp["pos"], inp["inv_freq"], inp["eps"])
    outs.update(q_out=qo, k_out=ko)
    grads += [inp["gq"], inp["gk"]]
    leaves.update(dq=q, dk=k, dwq=wq, dwk=wk)
    res = torch.autograd.grad(list(outs.values()), list(leaves.values()), grads)
    return outs, dict(zip(leaves, res))


# ------------------------------------------------------------- checks
def check_step(name: str, inp, bloth, dev, dist, world: int, rank: int, rows: range,
               seed: int, n_sample: int = 64) -> dict:
    """Checks one step of this rank's shard, outside any timed region.

    Tokens are independent, so `n_sample` sampled tokens of the shard are
    checked against the CPU oracle (float64) at the path's tolerance (bf16:
    abs <= 2e-2 or rel <= 1.6e-2). Weight gradients sum over every token of
    the batch: each rank's dweight (in the weight's dtype) is summed over the
    ranks by one all-reduce, and rank 0 compares the sum with the float64
    oracle over the whole batch and, at N > 1, with the same kernels run over
    the whole batch on its GPU. Each rank's dweight is rounded to bf16 before
    the sum, so the bound on the sum is the bf16 rule applied to the sum of
    the parts' magnitudes. Returns the check's record (rank 0's view)."""
    import oracle
    from oracle.reference_path import tolerance_ok
    B, S, Hd, Hq, Hk, D, theta, eps, packed = WORKLOADS[name]
    bf = torch.bfloat16
    outs, grads = run_step(inp, bloth)
    torch.cuda.synchronize(dev)
    worst = 0.0
    ok = True

    def note(good, excess):
        nonlocal ok, worst
        ok = ok and bool(good)
        worst = max(worst, float(excess))

    # ---- sampled tokens against the CPU oracle
    b = len(rows)
    gen = torch.Generator().manual_seed(97 + rank)
    flat = torch.randperm(b * S, generator=gen)[:n_sample]
    bi, si = flat // S, flat % S
    sel = lambda t: t.detach()[bi.to(t.device), si.to(t.device)].cpu()  # noqa: E731
    if "x" in inp:
        w = inp["w"].detach().cpu()
        if "r" in inp:
            ry, rz, _, rdz, _ = oracle.add_rms_norm_fwd_bwd(sel(inp["x"]), sel(inp["r"]), w,
                                                            sel(inp["gy"]), sel(inp["gz"]), eps)
            checks = [(outs["y"], ry), (outs["z"], rz), (grads["dx"], rdz), (grads["dr"], rdz)]
        else:
            ry, _, rdx, _ = oracle.rms_norm_fwd_bwd(sel(inp["x"]), w, sel(inp["gy"]), eps)
            checks = [(outs["y"], ry), (grads["dx"], rdx)]
        for got, ref in checks:
            note(*tolerance_ok(sel(got), ref, bf))
    wq, wk = inp["wq"].detach().cpu(), inp["wk"].detach().cpu()
    if "cos_q" in inp:
        for key, H, wt in (("q", Hq, wq), ("k", Hk, wk)):
            rsel = ((bi * S + si)[:, None] * H + torch.arange(H)[None, :]).reshape(-1)
            rows2 = lambda t: t.detach().reshape(-1, t.shape[-1])[rsel.to(t.device)].cpu()  # noqa: E731
            ry, _, rdx, _ = oracle.norm_rope_table_fwd_bwd(
                rows2(inp[key]), wt, rows2(inp["cos_" + key]), rows2(inp["sin_" + key]),
                rows2(inp["g" + key]), eps)
            note(*tolerance_ok(rows2(outs[key + "_out"]), ry, bf))
            note(*tolerance_ok(rows2(grads["d" + key]), rdx, bf))
    else:
        ref = oracle.qk_norm_rope_fwd_bwd(
            sel(inp["q"])[None], sel(inp["k"])[None], wq, wk, sel(inp["gq"])[None],
            sel(inp["gk"])[None], sel(inp["pos"])[None], inp["inv_freq"].cpu(), eps)
        for key, got in (("q_out", outs["q_out"]), ("k_out", outs["k_out"]),
                         ("dq", grads["dq"]), ("dk", grads["dk"])):
            note(*tolerance_ok(sel(got)[None], ref[key], bf))

    # ---- weight gradients summed over the ranks
    dw_keys = [k for k in ("dw", "dwq", "dwk") if k in grads]
    local = torch.cat([grads[k].detach().float() for k in dw_keys])
    total, mag = local.clone(), local.abs()
    if dist is not None:
        dist.all_reduce(total)
        dist.all_reduce(mag)
    fault = bloth.device_fault()
    rec = {"sampled_tokens_per_rank": int(flat.numel()), "sampled_worst_excess": worst}
    # the batch rows of all ranks together: rank r holds rows r*b .. r*b+b-1
    union = range(0, world * b)
    if rank == 0:
        # float64 oracle over those rows, one batch row at a time
        ref = torch.zeros_like(total, dtype=torch.float64)
        for r in union:
            one = make_inputs(name, range(r, r + 1), dev, seed)
            parts = []
            if "x" in one:
                w64 = one["w"].to(torch.float64)
                if "r" in one:
                    parts.append(oracle.add_rms_norm_fwd_bwd(one["x"], one["r"], w64, one["gy"],
                                                             one["gz"], eps)[4])
                else:
                    parts.append(oracle.rms_norm_fwd_bwd(one["x"], w64, one["gy"], eps)[3])
            if "cos_q" in one:
                for key in ("q", "k"):
                    parts.append(oracle.norm_rope_table_fwd_bwd(
                        one[key].reshape(-1, D), one["w" + key].to(torch.float64),
                        one["cos_" + key], one["sin_" + key], one["g" + key].reshape(-1, D),
                        eps)[3])
            else:
                rr = oracle.qk_norm_rope_fwd_bwd(
                    one["q"], one["k"], one["wq"].to(torch.float64),
                    one["wk"].to(torch.float64), one["gq"], one["gk"], one["pos"],
                    one["inv_freq"], eps)
                parts += [rr["dwq"], rr["dwk"]]
            ref += torch.cat(parts)
            del one
        bound = torch.clamp(1.6e-2 * mag.double(), min=2e-2)
        err = (total.double() - ref).abs()
        rec["dweight_max_abs_err_vs_oracle"] = float(err.max())
        rec["dweight_ok_vs_oracle"] = bool((err <= bound).all())
        ok = ok and rec["dweight_ok_vs_oracle"]
        if world > 1:
            full = make_inputs(name, union, dev, seed)
            _, g1 = run_step(full, bloth)
            one_gpu = torch.cat([g1[k].detach().float() for k in dw_keys])
            err1 = (total.double() - one_gpu.double()).abs()
            rec["dweight_max_abs_err_vs_one_gpu"] = float(err1.max())
            rec["dweight_ok_vs_one_gpu"] = bool((err1 <= bound).all())
            ok = ok and rec["dweight_ok_vs_one_gpu"]
            del full, g1
        rec["dweight_bound"] = "abs <= max(2e-2, 1.6e-2 * sum over ranks of |dweight_rank|)"
    flag = torch.tensor([0.0 if ok else 1.0, float(fault)], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    rec["ok"] = bool(flag[0].item() == 0.0)
    rec["fault"] = int(flag[1].item())
    return rec


# ------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while running
    (written to a temporary file that is removed afterwards)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="bloth_clocks_", suffix=".csv")
            self.fh = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or self.path is None or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as fh:
            for line in fh:
                f = [c.strip() for c in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- CPU arm
def cpu_port_step(name: str, tokens: int, seed: int = 0):
    """The oracle (float32, the reference golden's precision) fwd+bwd over
    `tokens` tokens of the workload; returns a callable running one step."""
    import oracle
    B, S, Hd, Hq, Hk, D, theta, eps, packed = WORKLOADS[name]
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    t = tokens
    x = torch.randn(t, Hd, generator=g).to(bf) if Hd else None
    w = (1 + 0.1 * torch.randn(Hd, generator=g)).to(bf) if Hd else None
    gy = torch.randn(t, Hd, generator=g).to(bf) if Hd else None
    res = name in RESIDUAL
    r = torch.randn(t, Hd, generator=g).to(bf) if res else None
    gz = torch.randn(t, Hd, generator=g).to(bf) if res else None
    q = torch.randn(1, t, Hq, D, generator=g).to(bf)
    k = torch.randn(1, t, Hk, D, generator=g).to(bf)
    wq = (1 + 0.1 * torch.randn(D, generator=g)).to(bf)
    wk = (1 + 0.1 * torch.randn(D, generator=g)).to(bf)
    gq = torch.randn(1, t, Hq, D, generator=g).to(bf)
    gk = torch.randn(1, t, Hk, D, generator=g).to(bf)
    pos = torch.arange(t) % S
    inv = oracle.inv_freq(D, theta)
    f32 = torch.float32

    tables = None
    if name in ROWS:  # per-row bf16 tables, expanded across heads
        ang = pos.to(f32)[:, None] * inv
        tables = {key: [getattr(torch, fn)(ang).to(bf)[:, None, :].expand(t, H, D // 2)
                        .reshape(-1, D // 2) for fn in ("cos", "sin")]
                  for key, H in (("q", Hq), ("k", Hk))}

    def step():
        if res:
            oracle.add_rms_norm_fwd_bwd(x, r, w, gy, gz, eps, compute=f32)
        elif Hd:
            oracle.rms_norm_fwd_bwd(x, w, gy, eps, compute=f32)
        if tables is not None:
            for rows, wt, gr, key in ((q, wq, gq, "q"), (k, wk, gk, "k")):
                c, s_ = tables[key]
                oracle.norm_rope_table_fwd_bwd(rows.reshape(-1, D), wt, c, s_,
                                               gr.reshape(-1, D), eps, compute=f32)
        else:
            oracle.qk_norm_rope_fwd_bwd(q, k, wq, wk, gq, gk, pos.view(1, t), inv, eps,
                                        compute=f32)

    return step


def time_cpu(name: str, min_seconds: float = CPU_MIN_SECONDS, min_steps: int = 1,
             warmup: int = 1):
    """Times the oracle port on all host cores; returns (tokens/s, sample,
    cores, steps).

    Every step is the same fixed sample of CPU_SAMPLE_TOKENS tokens of the
    workload; steps run until both `min_steps` steps and `min_seconds`
    seconds are done, so the rate is averaged over at least that long."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    tokens = CPU_SAMPLE_TOKENS
    step = cpu_port_step(name, tokens)
    for _ in range(max(warmup, 1)):
        step()
    t0 = time.perf_counter()
    n = 0
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if n >= min_steps and el >= min_seconds:
            break
    sample = (f"{tokens} tokens of the workload per step (fixed sample), {n} steps, "
              f"{el:.1f} s, float32 oracle port on {cores} host threads")
    return tokens * n / el, sample, cores, n


# ------------------------------------------------------------- reference GPU
def reference_triton_step_ms(name: str, steps: int, warmup: int) -> dict:
    """The reference's own GPU kernels (Triton) on the same workload, one GPU:
    ``bloth.kernels.rms_norm`` on the hidden rows and
    ``bloth.kernels.fused_norm_rope`` on the q and k head rows, forward and
    backward, from the reference package installed under baseline/_ref. Its
    fused contract takes one cos/sin row per normalised row, so the tables
    are expanded across heads (bf16, as BlothRoPE caches them) before the
    timed region: that work is not timed, in the reference's favour. Its
    fused backward omits the transposed rotation, so this is a speed
    reference only. Timed like the main arm: CUDA graphs of the step. The
    same step through this library's implementation of the same two entry
    points, on the same inputs, is timed beside it (``same_api_b200``)."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "bloth")):
        return {"unavailable": "reference not installed under baseline/_ref"}
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import bloth as ref  # noqa: F401
    from bloth.kernels import fused_norm_rope, rms_norm
    dev = torch.device("cuda", torch.cuda.current_device())
    B, S, Hd, Hq, Hk, D, theta, eps, packed = WORKLOADS[name]
    inp = make_inputs(name, B, dev, seed=1234)
    ang = inp["pos"].to(torch.float32).unsqueeze(-1) * inp["inv_freq"]  # [B, S, D/2]
    tabs = {}
    for key, H in (("q", Hq), ("k", Hk)):
        c = torch.cos(ang).to(torch.bfloat16).unsqueeze(2).expand(B, S, H, D // 2)
        s_ = torch.sin(ang).to(torch.bfloat16).unsqueeze(2).expand(B, S, H, D // 2)
        tabs[key] = (c.reshape(-1, D // 2).contiguous(), s_.reshape(-1, D // 2).contiguous())

    def step(norm, fused):
        outs, grads, leaves = [], [], []
        if Hd:
            x = inp["x"].requires_grad_(True)
            w = inp["w"].requires_grad_(True)
            outs.append(norm(x, w, eps))
            grads.append(inp["gy"])
            leaves += [x, w]
        for key, wkey, gkey in (("q", "wq", "gq"), ("k", "wk", "gk")):
            t = inp[key].view(-1, D).requires_grad_(True)
            w = inp[wkey].requires_grad_(True)
            outs.append(fused(t, w, tabs[key][0], tabs[key][1], eps))
            grads.append(inp[gkey].view(-1, D))
            leaves += [t, w]
        return torch.autograd.grad(outs, leaves, grads)

    def time_step(norm, fused):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(max(warmup, 3)):
                step(norm, fused)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        unroll = next(u for u in (20, 10, 8, 5, 4, 2, 1) if steps % u == 0)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(unroll):
                step(norm, fused)
        replays = max(1, steps // unroll)
        graph.replay()
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(replays):
            graph.replay()
        end.record()
        torch.cuda.synchronize(dev)
        del graph
        return start.elapsed_time(end) / (replays * unroll), replays * unroll

    ms_step, nsteps = time_step(rms_norm, fused_norm_rope)
    import bloth_b200
    ms_b200, _ = time_step(bloth_b200.rms_norm, bloth_b200.kernels.fused_norm_rope)
    tokens = B * S
    nbytes = step_bytes(tokens, name)["total"]
    del inp, tabs
    torch.cuda.empty_cache()
    return {"ms_per_step": ms_step, "tokens_per_s": tokens / (ms_step / 1e3),
            "steps": nsteps, "gbps": round(nbytes / (ms_step / 1e3) / 1e9, 1),
            "workload": describe(name),
            "note": "reference Triton kernels (rms_norm, fused_norm_rope per head row, "
                    "per-row bf16 cos/sin tables expanded before timing), CUDA graphs",
            "same_api_b200": {"ms_per_step": ms_b200, "tokens_per_s": tokens / (ms_b200 / 1e3),
                              "note": "bloth_b200.rms_norm and "
                                      "bloth_b200.kernels.fused_norm_rope on the same inputs "
                                      "and per-row tables"}}


# ------------------------------------------------------------- main
def run_config(name: str, tokens_local: int, world: int, scaling: str, peak: float,
               nbytes: dict | None = None, gbps: float | None = None) -> dict:
    """The config object both arms print (same keys, so the lines compare)."""
    cfg = {"workload": describe(name), "tokens_per_gpu": tokens_local, "scaling": scaling,
           "parallelism": f"{world} independent row shard{'s' if world > 1 else ''}, "
                          "no collective",
           "l2": "inputs larger than L2 (each tensor >= 67 MB at 32768 tokens; at smaller "
                 "shards the step's working set still exceeds the 126 MB L2), no flush",
           "step_gb_per_gpu": round(step_bytes(tokens_local, name)["total"] / 1e9, 4)}
    if gbps is not None:
        cfg["gbps"] = round(gbps, 1)
        cfg["frac_of_8tbs_per_gpu"] = round(gbps / world / NOMINAL_HBM_GBS, 4)
        cfg["frac_of_measured_per_gpu"] = round(gbps / world / peak, 4)
    return cfg


def stream_ceilings(dev, mib: int = 256, reps: int = 8) -> dict:
    """Streaming rates of this GPU during the run, beside the roofline: a
    1-read:1-write copy and a 2-read:1-write add into a third tensor (the
    traffic mixes of the forward and the backward kernels), bf16, `mib` MiB per
    tensor (each beyond the 126 MB L2), torch's own kernels in a CUDA graph of
    10 operations, median of `reps` replays."""
    n = mib * 2**20 // 2
    x = torch.ones(n, device=dev, dtype=torch.bfloat16)
    y = torch.ones_like(x)
    z = torch.empty_like(x)
    out = {"tensor_mib": mib}
    for key, fn, moved in (("copy_1r1w_gbs", lambda: y.copy_(x), 2 * n * 2),
                           ("add_2r1w_gbs", lambda: torch.add(x, y, out=z), 3 * n * 2)):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(10):
                fn()
        g.replay()
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b) / 10)
        times.sort()
        out[key] = round(moved / (times[len(times) // 2] / 1e3) / 1e9, 1)
        del g
    del x, y, z
    torch.cuda.empty_cache()
    return out


def measured_peak() -> tuple[float, bool]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), True
    except (OSError, KeyError, ValueError):
        return 6650.0, False


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="llama3-8b", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-triton"])
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="default: strong for the sharded workloads (llama3-8b, "
                         "qwen3-8b-packed), weak otherwise")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="on one GPU, run the shard rank 0 of an N-rank strong-scaling job "
                         "processes")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=CPU_MIN_SECONDS)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the post-run parity check (profiling runs)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's Triton kernels beside the main line")
    ap.add_argument("--sweep", action="store_true",
                    help="bandwidth sweep over token counts 2^14..2^24 (hidden 8192 and "
                         "32q/8k heads of 128, bf16 and fp32; chunked above the resident "
                         "sizes); prints one JSON line, one GPU")
    ap.add_argument("--sweep-point", default=None,
                    help="with --sweep, run only the points DTYPE:LG:OP (e.g. float32:16:qk; "
                         "any field may be '*'): a fixed launch sequence for profilers")
    ap.add_argument("--once", action="store_true",
                    help="run --warmup steps and one more fwd+bwd step, untimed, and exit "
                         "(a fixed launch sequence for profilers)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    name = args.workload
    B, S, Hd, Hq, Hk, D, theta, eps, packed = WORKLOADS[name]
    scaling = args.scaling or default_scaling(name)
    if args.shard_of > 1 and world > 1:
        raise SystemExit("bench.py: --shard-of emulates one rank on one GPU; do not combine "
                         "it with torchrun")
    shards = max(world, args.shard_of)
    peak, peak_measured = measured_peak()

    if args.impl == "reference":
        if rank != 0:
            return
        tps, sample, cores, n = time_cpu(name, args.cpu_seconds, min_steps=1,
                                        warmup=min(max(args.warmup, 1), 3))
        tokens_local = local_batch(B, shards, scaling) * S
        line = {"metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": n, "warmup": args.warmup, "impl": "reference",
                "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": run_config(name, tokens_local, world, scaling, peak),
                "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores,
                                 "kind": "port", "sample": sample},
                "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if args.sweep or args.sweep_point:
        sweep(args, world, rank, local)
        return

    if args.impl == "reference-triton":
        if rank == 0:
            torch.cuda.set_device(local)
            rec = reference_triton_step_ms(name, args.steps, args.warmup)
            print(json.dumps({"metric": METRIC, "impl": "reference-triton", **rec}), flush=True)
        return

    import bloth_b200 as bloth
    from bloth_b200 import _lib

    if not torch.cuda.is_available():
        raise SystemExit("bench.py: no CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    # this rank's shard of batch rows (tokens_local tokens per step)
    rows = shard_rows(B, shards, rank, scaling)
    tokens_local = len(rows) * S
    seed = 1234
    inp = make_inputs(name, rows, dev, seed=seed)
    nbytes = step_bytes(tokens_local, name)
    if args.once:
        for _ in range(args.warmup + 1):
            run_step(inp, bloth)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.destroy_process_group()
        return
    bloth.device_fault(reset=True)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- one fwd+bwd step through the public API, captured as CUDA graphs of
    # UNROLL steps; replaying a graph runs every kernel of every step without
    # host gaps. Graph A (warm-up) has an event pair around every C-ABI launch
    # of its last step: the per-kernel breakdown, and which call dominates.
    # Graph B (timed) has event pairs only around the dominant call, in every
    # fifth step, so that instrumentation adds little to the timed steps.
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            run_step(inp, bloth)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    # kernels one step launches, counted by the library itself
    n0 = bloth.kernel_launch_count()
    run_step(inp, bloth)
    launches_per_step = bloth.kernel_launch_count() - n0
    torch.cuda.synchronize(dev)
    unroll = next(u for u in (20, 10, 8, 5, 4, 2, 1) if args.steps % u == 0)  # exactly K steps
    every = 5 if unroll % 5 == 0 else 1

    def capture(timed_steps, only=None):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(unroll):
                if i in timed_steps:
                    with _lib.timing_launches(external=True, only=only) as tm:
                        run_step(inp, bloth)
                    timers.append(tm)
                else:
                    run_step(inp, bloth)
        return g

    timers = []
    n_inst = min(5, unroll)  # instrumented steps at the end of the warm-up graph
    graph_a = capture(set(range(unroll - n_inst, unroll)))
    for _ in range(max(1, args.warmup // unroll)):
        graph_a.replay()
    barrier()
    per_kernel = merge_summaries([tm.summary() for tm in timers])
    dominant = max(per_kernel.items(), key=lambda kv: kv[1]["total_ms"])[0]
    del graph_a
    timers = []
    graph = capture({i for i in range(unroll) if (i + 1) % every == 0}, only={dominant})
    replays = max(1, args.steps // unroll)
    steps = replays * unroll
    graph.replay()
    barrier()

    # ---- device-resident timed region
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        start.record()
        for _ in range(replays):
            graph.replay()
        end.record()
        barrier()
    ms = max_over_ranks(start.elapsed_time(end), dist, dev)
    # the dominant call's time per step (summed over its launches in the step:
    # the table contract calls it once for q and once for k): its event pairs
    # re-record on every replay, so they are read after the timed region's
    # last replay and after each of a few more replays of the same graph,
    # and the median over all of those instrumented steps is taken
    def dominant_times():
        return [sum(a.elapsed_time(b) for a, b in tm.pairs[dominant]) for tm in timers]

    dom_all = dominant_times()
    for _ in range(15):
        graph.replay()
        torch.cuda.synchronize(dev)
        dom_all += dominant_times()
    dom_all.sort()
    dom_ms = dom_all[len(dom_all) // 2]
    del graph
    ms_step = ms / steps
    tokens_total = tokens_local * world
    value = tokens_total / (ms_step / 1e3)
    gbps = nbytes["total"] * world / (ms_step / 1e3) / 1e9
    # the fault word after the timed replays (an expired copy wait anywhere
    # in them would show here)
    fault_timed = int(max_over_ranks(float(bloth.device_fault()), dist, dev))

    # the same step called eagerly from Python (host launch overhead included)
    eager_steps = min(200, steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for _ in range(eager_steps):
        run_step(inp, bloth)
    e1.record()
    barrier()
    eager_ms = max_over_ranks(e0.elapsed_time(e1), dist, dev) / eager_steps

    launches = launches_per_step * steps
    kb = {"bloth_rmsnorm_fwd": "rms_fwd", "bloth_rmsnorm_bwd": "rms_bwd",
          "bloth_add_rmsnorm_fwd": "add_fwd", "bloth_add_rmsnorm_bwd": "add_bwd",
          "bloth_qk_norm_rope_fwd": "qk_fwd", "bloth_qk_norm_rope_bwd": "qk_bwd",
          "bloth_norm_rope_fwd": "nr_fwd", "bloth_norm_rope_bwd": "nr_bwd"}
    top_bytes = nbytes[kb[dominant]]
    achieved = top_bytes / (dom_ms / 1e3) / 1e9
    kernels = {k: {"launches": v["launches"], "mean_us": round(v["mean_ms"] * 1e3, 2),
                   "gbps": round(nbytes[kb[k]] / (v["total_ms"] / 1e3) / 1e9, 1)}
               for k, v in per_kernel.items()}
    traffic = PROFILED_TRAFFIC.get((name, dominant)) if tokens_local == 32768 else None

    # ---- results checked outside the timed region (every rank)
    check = None
    if not args.no_check:
        check = check_step(name, inp, bloth, dev, dist, world, rank, rows, seed)

    # ---- end to end through the public API with host buffers
    e2e = None
    if args.e2e_steps > 0:
        e2e = end_to_end(inp, bloth, dev, args.e2e_steps, barrier, dist, tokens_total)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tps, sample, cores, _ = time_cpu(name, args.cpu_seconds)
        cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": sample}

    ref_gpu = None
    if rank == 0 and world == 1 and args.shard_of == 1 and not args.no_reference_gpu:
        del inp
        torch.cuda.empty_cache()
        try:
            ref_gpu = reference_triton_step_ms(name, min(args.steps, 200), 3)
        except Exception as exc:  # noqa: BLE001 - reported, never fatal to the main line
            ref_gpu = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}

    # the GPU's own streaming rates in this run, for the roofline's context
    ceil = stream_ceilings(dev) if rank == 0 else None

    if rank == 0:
        cfg = run_config(name, tokens_local, world, scaling, peak, nbytes, gbps)
        if args.shard_of > 1:
            cfg["emulated_shard_of"] = args.shard_of
        cfg.update({
            "timing": f"CUDA graph of {unroll} steps through the public API, "
                      f"{replays} replays; event pairs around the dominant call "
                      f"in every {every}th step (roofline, median of {len(dom_all)}); the "
                      f"per-kernel breakdown below is the median over {n_inst} instrumented "
                      "warm-up steps",
            "eager_ms_per_step": round(eager_ms, 4),
            "per_gpu_tokens_per_s": round(value / world),
            "kernels": kernels,
            "launches_per_step": launches_per_step})
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": cfg,
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"
                         if peak_measured else "fallback 6650 GB/s (of fallback)",
                         "traffic": traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                           "profiles/ (cold-L2 single launch at 32768 tokens)",
                         # the same call against the streaming rate of its own
                         # traffic mix measured in this run (backward calls read
                         # two tensors per one written, forward calls one)
                         "stream_ceilings": ceil,
                         "frac_of_stream_ceiling": round(
                             achieved / ceil["add_2r1w_gbs" if dominant.endswith("_bwd")
                                             else "copy_1r1w_gbs"], 4)},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "fault": max(fault_timed, check["fault"] if check else 0),
            "parity_ok": None if check is None else check["ok"],
            "parity": check,
            "reference_gpu": ref_gpu,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def sweep(args, world: int = 1, rank: int = 0, local: int = 0) -> None:
    """fwd+bwd GB/s of the hidden RMSNorm (rows of 8192) and of the q/k pair
    (32 + 8 heads of 128, positions in-register) at token counts 2^14 .. 2^24,
    bf16 and fp32, each op alone in a CUDA graph of 10 steps. Tensors stay
    resident up to 2^20 tokens (bf16) / 2^18 (fp32) per GPU, where one op
    holds ~40-70 GB of HBM. Larger counts (a hidden fp32 tensor at 2^24 tokens
    is 550 GB) run chunked, as rows are independent: chunks of the largest
    resident size through the same device buffers, in a graph of one such
    step. Every chunk's tensors are many times the L2 size, so reusing the
    buffers saves no traffic. Inputs ~N(0, 1); rates do not depend on the
    values. Under torch.distributed.run each point's tokens are split over
    the ranks (strong scaling, no collective in the timed region); its time
    is the max over ranks and its rate the whole job's."""
    import bloth_b200 as bloth
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    peak, _ = measured_peak()
    Hd, Hq, Hk, D = 8192, 32, 8, 128
    inv = (1.0 / (5e5 ** (torch.arange(0, D // 2, dtype=torch.float32) / (D // 2)))).to(dev)
    points = []
    want = (args.sweep_point or "*:*:*").split(":")
    if len(want) != 3:
        raise SystemExit("--sweep-point takes DTYPE:LG:OP")

    def wanted(dt, lg, op):
        return all(w in ("*", v) for w, v in zip(want, (str(dt).replace("torch.", ""),
                                                        str(lg), op)))

    for dt, top in ((torch.bfloat16, 20), (torch.float32, 18)):
        s = torch.tensor([], dtype=dt).element_size()
        for lg in range(14, 25, 2):
            lw = world.bit_length() - 1  # world is a power of two (1, 2, 4, 8)
            nchunk = 1 << max(0, lg - lw - top)  # chunks of the largest resident size
            T = (1 << lg) // world // nchunk  # tokens of one rank's chunk
            g = torch.Generator(device=dev).manual_seed(min(lg, top))
            for op in ("hidden", "qk"):
                if not wanted(dt, lg, op):
                    continue
                if op == "hidden":
                    x = torch.randn(T, Hd, generator=g, device=dev, dtype=dt).requires_grad_(True)
                    w = torch.ones(Hd, device=dev, dtype=dt).requires_grad_(True)
                    gy = torch.randn(T, Hd, generator=g, device=dev, dtype=dt)
                    nbytes = T * (5 * Hd * s + 8)

                    def one():
                        return torch.autograd.grad(bloth.rms_norm(x, w, 1e-6), (x, w), gy)
                else:
                    q = torch.randn(1, T, Hq, D, generator=g, device=dev,
                                    dtype=dt).requires_grad_(True)
                    k = torch.randn(1, T, Hk, D, generator=g, device=dev,
                                    dtype=dt).requires_grad_(True)
                    wq = torch.ones(D, device=dev, dtype=dt).requires_grad_(True)
                    wk = torch.ones(D, device=dev, dtype=dt).requires_grad_(True)
                    gq, gk = torch.randn_like(q), torch.randn_like(k)
                    pos = (torch.arange(T, device=dev) % 8192).view(1, T)
                    nbytes = T * ((Hq + Hk) * (5 * D * s + 8) + 16)

                    def one():
                        out = bloth.fused_qk_norm_rope(q, k, wq, wk, pos, inv, 1e-6)
                        return torch.autograd.grad(out, (q, k, wq, wk), (gq, gk))

                def step():
                    for _ in range(nchunk):
                        one()
                nbytes *= nchunk
                unroll = 10 if nchunk == 1 else 1
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    for _ in range(3):
                        step()
                torch.cuda.current_stream(dev).wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for _ in range(unroll):
                        step()
                graph.replay()
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = 3 if T >= (1 << 18) else 20
                if dist is not None:
                    dist.barrier()
                    torch.cuda.synchronize(dev)
                e0.record()
                for _ in range(reps):
                    graph.replay()
                e1.record()
                torch.cuda.synchronize(dev)
                ms = max_over_ranks(e0.elapsed_time(e1) / (unroll * reps), dist, dev)
                nbytes *= world
                gbps = nbytes / (ms / 1e3) / 1e9
                total = T * nchunk * world
                points.append({"tokens": total, "dtype": str(dt).replace("torch.", ""), "op": op,
                               "gpus": world, "chunks": nchunk, "ms_fwd_bwd": round(ms, 4),
                               "gbps": round(gbps, 1),
                               "frac_of_measured_per_gpu": round(gbps / world / peak, 4),
                               "tokens_per_s": round(total / (ms / 1e3))})
                del graph
                if op == "hidden":
                    del x, w, gy
                else:
                    del q, k, wq, wk, gq, gk
                torch.cuda.empty_cache()
    fault = int(max_over_ranks(float(bloth.device_fault()), dist, dev))
    if rank == 0:
        print(json.dumps({"sweep": f"fwd+bwd bandwidth vs size, {world} B200"
                                   f"{'s, tokens split over the ranks' if world > 1 else ''}",
                          "peak_gbs": peak, "fault": fault, "points": points}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def end_to_end(inp, bloth, dev, steps, barrier, dist, tokens_total):
    """The same step through the public API with every input in pinned host
    memory: each step copies its inputs host->device and all of its results
    (outputs and gradients) device->host inside the timed region. Transfers
    are pipelined as a streaming user would: step i+1's inputs upload on a
    copy stream while step i computes, and step i's results download on a
    third stream (two device input buffers; events order every reuse)."""
    keys_in = [k for k in ("x", "r", "gy", "gz", "q", "k", "gq", "gk", "pos", "cos_q", "sin_q",
                           "cos_k", "sin_k") if k in inp]
    host = {k: inp[k].detach().cpu().pin_memory() for k in keys_in}
    small = {k: v for k, v in inp.items() if k not in keys_in}
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    bufs = [{k: torch.empty_like(inp[k]) for k in keys_in} for _ in range(2)]
    s_main = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    outs_host = None

    def upload(i):
        b = bufs[i % 2]
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_free[i % 2])  # step i-2 has finished reading this buffer
            for k in keys_in:
                b[k].copy_(host[k], non_blocking=True)
            ev_in[i % 2].record(s_in)

    def compute_and_download(i):
        nonlocal outs_host
        b = bufs[i % 2]
        s_main.wait_event(ev_in[i % 2])
        d = {k: b[k].detach() for k in keys_in}
        d.update(small)
        outs, grads = run_step(d, bloth)
        ev_free[i % 2].record(s_main)
        res = [t.detach() for t in list(outs.values()) + list(grads.values())]
        if outs_host is None:
            outs_host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in res]
        s_out.wait_stream(s_main)
        with torch.cuda.stream(s_out):
            for h, t in zip(outs_host, res):
                t.record_stream(s_out)
                h.copy_(t, non_blocking=True)

    # warm-up pass of the whole pipeline
    upload(0)
    compute_and_download(0)
    torch.cuda.synchronize(dev)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_main)
    s_in.wait_stream(s_main)
    upload(0)
    for i in range(steps):
        if i + 1 < steps:
            upload(i + 1)
        compute_and_download(i)
    s_main.wait_stream(s_out)
    end.record(s_main)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end), dist, dev)
    d2h = sum(t.numel() * t.element_size() for t in outs_host)

    # the same transfers alone (uploads on one stream, downloads of as many
    # bytes on another, overlapped): the PCIe time the step cannot beat
    dev_out = [torch.empty(h.shape, dtype=h.dtype, device=dev) for h in outs_host]
    barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(s_main)
    s_in.wait_stream(s_main)
    s_out.wait_stream(s_main)
    for i in range(steps):
        with torch.cuda.stream(s_in):
            for k in keys_in:
                bufs[i % 2][k].copy_(host[k], non_blocking=True)
        with torch.cuda.stream(s_out):
            for h, t in zip(outs_host, dev_out):
                h.copy_(t, non_blocking=True)
    s_main.wait_stream(s_in)
    s_main.wait_stream(s_out)
    c1.record(s_main)
    barrier()
    copy_ms = max_over_ranks(c0.elapsed_time(c1), dist, dev)
    return {"value": tokens_total / (ms / steps / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms / steps,
            "transfers_only_ms_per_step": copy_ms / steps,
            "h2d_plus_d2h_gbs": round((h2d + d2h) / (copy_ms / steps / 1e3) / 1e9, 1)}


if __name__ == "__main__":
    main()
