"""The bench's roofline model: algorithmic bytes/flops per benchmark workload."""

import bench


def test_config2_bytes_and_flops():
    # B2 T4096 H16 K=V=128 bf16 with h0: 1032 B per token-head + 2 states per (b,h)
    assert bench.algo_bytes(2, 4096, 16, h0=True) == 139_460_608
    assert bench.algo_flops(2, 4096, 16) == 2 * 4096 * 16 * 163_840


def test_roofline_time_config2():
    hbm, tf, _ = bench.load_peaks()
    t_hbm = bench.algo_bytes(2, 4096, 16) / (hbm * 1e9)
    t_tc = bench.algo_flops(2, 4096, 16) / (tf * 1e12)
    assert t_hbm > t_tc          # HBM binds at the headline shape
    assert 15e-6 < t_hbm < 30e-6


def test_reference_arm_line_shape():
    import argparse
    args = argparse.Namespace(gpus=1, steps=1, warmup=0, impl="reference", config=1, no_cpu_baseline=False)
    cfg = dict(bench.CONFIGS[1])
    cfg["T"] = 128  # tiny sample for the test
    line = bench.run_reference(args, cfg, rank=0, world=1)
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
    assert bench.run_reference(args, cfg, rank=1, world=2) is None
