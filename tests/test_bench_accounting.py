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
