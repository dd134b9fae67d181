"""bench.py host logic on the CPU: the byte model and the synthetic inputs of
the workloads, in particular the reference-contract one (q and k as rows with
per-row cos/sin tables), and the CPU port that times them."""
import math

import torch

import bench


def test_rows_workload_bytes_add_the_tables_and_drop_the_positions():
    tokens = 32768
    pos_path = bench.step_bytes(tokens, "llama3-8b")
    rows_path = bench.step_bytes(tokens, "llama3-8b-rows")
    assert rows_path["rms_fwd"] == pos_path["rms_fwd"]
    assert rows_path["rms_bwd"] == pos_path["rms_bwd"]
    # per head row and pass: cos + sin rows of 64 bf16 = 256 B; positions 8 B per token and pass
    heads = 32 + 8
    assert rows_path["total"] - pos_path["total"] == tokens * (heads * 2 * 256 - 16)
    assert rows_path["nr_fwd"] == tokens * heads * (2 * 128 * 2 + 4 + 256)
    assert rows_path["nr_bwd"] == tokens * heads * (3 * 128 * 2 + 4 + 256)
    assert abs(rows_path["total"] / 1e9 - 3.7017) < 1e-3


def test_rows_workload_tables_follow_the_positions():
    inp = bench.make_inputs("llama3-8b-rows", 1, torch.device("cpu"), seed=0)
    S, Hq, Hk, half = 4096, 32, 8, 64
    assert inp["cos_q"].shape == (S * Hq, half) and inp["sin_k"].shape == (S * Hk, half)
    assert inp["cos_q"].dtype == torch.bfloat16 and inp["cos_q"].is_contiguous()
    inv = inp["inv_freq"]
    for s, h in ((0, 0), (7, 31), (4095, 5)):
        ang = float(s) * inv
        assert torch.equal(inp["cos_q"][s * Hq + h], torch.cos(ang).to(torch.bfloat16))
        assert torch.equal(inp["sin_q"][s * Hq + h], torch.sin(ang).to(torch.bfloat16))
        kh = h % Hk
        assert torch.equal(inp["cos_k"][s * Hk + kh], torch.cos(ang).to(torch.bfloat16))
    assert math.isclose(float(inv[1]), 1.0 / (5e5 ** (1 / 64)), rel_tol=1e-6)


def test_cpu_port_runs_every_workload():
    for name in bench.WORKLOADS:
        bench.cpu_port_step(name, 16)()
    assert "fused_norm_rope" in bench.describe("llama3-8b-rows")


def test_shards_hold_exactly_the_rows_of_the_whole_batch(monkeypatch):
    # every batch row is seeded on its own, so the union of the ranks' shards
    # is the unsharded batch, wherever each shard is generated (a small
    # packed workload with the layout of the Qwen3 one)
    cpu = torch.device("cpu")
    name = "tiny-packed"
    monkeypatch.setitem(bench.WORKLOADS, name, (8, 3000, 64, 4, 2, 64, 1e6, 1e-6, True))
    B = bench.WORKLOADS[name][0]
    full = bench.make_inputs(name, range(B), cpu)
    for world in (2, 4, 8):
        for rank in range(world):
            rows = bench.shard_rows(B, world, rank, "strong")
            part = bench.make_inputs(name, rows, cpu)
            sl = slice(rows.start, rows.stop)
            for key in ("x", "gy", "q", "k", "gq", "gk", "pos"):
                assert torch.equal(part[key], full[key][sl]), (world, rank, key)
            for key in ("w", "wq", "wk", "inv_freq"):
                assert torch.equal(part[key], full[key])
    # weak scaling: every rank runs a full batch of its own rows
    assert bench.shard_rows(8, 4, 3, "weak") == range(24, 32)


def test_sharded_workloads_default_to_strong_scaling():
    assert bench.default_scaling("llama3-8b") == "strong"
    assert bench.default_scaling("qwen3-8b-packed") == "strong"
    assert bench.default_scaling("llama3.2-1b") == "weak"
    assert bench.local_batch(8, 8, "strong") * 4096 == 4096


def test_per_kernel_breakdown_is_the_median_over_instrumented_steps():
    steps = [{"bloth_rmsnorm_bwd": {"launches": 2, "total_ms": t, "mean_ms": t / 2}}
             for t in (0.140, 0.131, 0.500, 0.129, 0.135)]
    got = bench.merge_summaries(steps)["bloth_rmsnorm_bwd"]
    assert got["launches"] == 2
    assert got["total_ms"] == 0.135 and got["mean_ms"] == 0.135 / 2
