"""bench.py's algorithmic work accounting (CPU): the per-step flop count and the
per-stage units that the roofline divides by kernel time, for MHA and for
grouped-query heads (attention work per query head, solve work per kv head)."""
import bench


def test_flops_per_step_mha_is_14_n2d_per_head():
    B, H, N, D = 1, 32, 32768, 128
    assert bench.flops_per_step(B, H, N, D) == 14.0 * N * N * D * B * H
    assert bench.flops_per_step(B, H, N, D, H) == bench.flops_per_step(B, H, N, D)
    # the headline: 61.6 TFLOP per step
    assert abs(bench.flops_per_step(B, H, N, D) / 1e12 - 61.57) < 0.01


def test_flops_per_step_gqa():
    B, Hq, Hkv, N, D = 1, 32, 4, 32768, 128
    fl = bench.flops_per_step(B, Hq, N, D, Hkv)
    assert fl == 7.0 * N * N * D * (Hq + Hkv)
    assert abs(fl / 1e12 - 34.6) < 0.05


def test_stage_units_sum_to_the_step():
    for H, Hkv in ((32, 32), (32, 4), (8, 1)):
        u = bench.stage_units(H, Hkv)
        # 7 N^2 D of attention per query head and 7 of solve per kv head
        assert sum(u.values()) == 7 * (H + Hkv)
        assert u["attn_fwd"] + u["attn_bwd"] + u["attn_bwd_row"] == 7 * H
        assert u["solve_fwd"] + u["solve_bwd"] + u["solve_bwd_row"] == 7 * Hkv


def test_gqa_config_is_registered():
    B, H, N, D, _ = bench.CONFIGS["32k-gqa"]
    assert (B, H, N, D) == (1, 32, 32768, 128) and bench.KV_HEADS["32k-gqa"] == 4
    assert all(bench.KV_HEADS.get(c, bench.CONFIGS[c][1]) == bench.CONFIGS[c][1]
               for c in ("32k", "cfg2", "small", "8k"))


def test_shard_splits_the_whole_job():
    # the metric's configuration: 32 heads over 1/2/4/8 ranks, contiguous kv heads
    for W in (1, 2, 4, 8):
        got = [bench.shard(1, 32, W, r) for r in range(W)]
        assert all(g == (0, 1, r * 32 // W, 32 // W) for r, g in enumerate(got))
    # config 2: B4 H32 -> 16 (batch, head) pairs per GPU at 8 GPUs, whole batch elements below
    assert bench.shard(4, 32, 8, 3) == (1, 1, 16, 16)
    assert bench.shard(4, 32, 2, 1) == (2, 2, 0, 32)
    assert bench.shard(4, 32, 4, 2) == (2, 1, 0, 32)
    # config 3 (LUCID-Path B2 H16): 4 pairs per GPU at 8 GPUs
    assert bench.shard(2, 16, 8, 5) == (1, 1, 4, 4)
    # every pair exactly once
    for B, H, W in ((4, 32, 8), (2, 16, 4), (1, 4, 2)):
        seen = set()
        for r in range(W):
            b0, nb, h0, nh = bench.shard(B, H, W, r)
            seen |= {(b, h) for b in range(b0, b0 + nb) for h in range(h0, h0 + nh)}
        assert len(seen) == B * H
    import pytest
    with pytest.raises(ValueError):
        bench.shard(1, 4, 8, 0)          # 4 kv heads (the GQA layout) cannot split over 8 ranks


def test_peak_fraction_divides_by_all_gpus():
    """The line's frac_of_bf16_peak is the whole-job rate over the peak of every GPU."""
    import inspect
    src = inspect.getsource(bench.bench_lucid) + inspect.getsource(bench.bench_path)
    assert src.count("tflops / (pk_sust * world)") == 2
