"""bench.py's host-side pieces on the CPU: the per-config summary of the JSON line and the CPU arms' restated
reference paths at tiny sizes (no GPU involved)."""

import json

import bench


def _line():
    c3 = {k: {"tflops": 2000.0, "frac_fp8_peak": 0.44} for k in ("linear_3072", "gate_up_16384", "down_3072_k8192")}
    return {
        "value": 3700.0, "n_gpus": 2, "device_status": 0,
        "roofline": {"frac": 0.45},
        "e2e": {"value": 820.0, "host_link": {"h2d_gbs_per_rank": 52.0, "both_gbs_per_rank": 54.0}},
        "configs": {
            "configs[0]": {"gemm_us": 29.7, "gemm_tflops": 2600.0, "gemm_frac_fp4_peak": 0.29, "quant_us": 12.3,
                           "linear_tflops": 1900.0, "e2e": {"tflops": 81.0}},
            "configs[2]": {"adaln_quant_gbs": 1850.0, "adaln_quant_frac_hbm": 0.29, "rms_rope_qkv_gbs": 4960.0,
                           "rms_rope_qkv_frac_hbm": 0.77},
            "configs[3]": c3},
        "dit": {"step_ms_at_4096_tokens": 13.5, "img_per_s": 6.2,
                "tensor_parallel_latency": {"world": 2, "step_ms": 13.3, "step_ms_nccl": 14.6}},
        "cpu_baseline": {"value": 0.2},
        "cpu_baseline_configs0_3": {"c0_nvfp4_tflops": 0.26, "c3_fp8_tflops": 0.21},
    }


def test_summary_carries_every_config():
    s = bench.summary(_line())
    assert s["c1_mlp_tflops"] == 3700.0 and s["c1_e2e_tflops"] == 820.0 and s["c1_gu_frac_fp4"] == 0.45
    assert s["c0_gemm_us"] == 29.7 and s["c0_e2e_tflops"] == 81.0
    assert s["c3_fp8_tflops"] == [2000.0] * 3
    assert s["c4_img_per_s_per_gpu"] == 3.1 and s["c4_tp_world"] == 2
    assert s["cpu_c0_tflops"] == 0.26 and s["cpu_c3_fp8_tflops"] == 0.21
    assert s["link_both_gbs"] == 54.0 and s["device_status"] == 0
    json.dumps(s)


def test_summary_without_optional_legs():
    line = _line()
    for k in ("configs", "dit", "cpu_baseline", "cpu_baseline_configs0_3"):
        line.pop(k)
    s = bench.summary(line)
    assert "c0_gemm_us" not in s and "c4_step_ms" not in s and s["c1_mlp_tflops"] == 3700.0


def test_cpu_arms_small():
    """The CPU arms at a few rows: positive rates, thread count and sample described."""
    r = bench.cpu_baseline_linears(budget_s=0.05, rows=4)
    assert r["c0_nvfp4_tflops"] > 0 and r["c3_fp8_tflops"] > 0 and r["cores"] >= 1 and r["kind"] == "port"
    f = bench.cpu_baseline_fusions(budget_s=0.05, rows=8)
    assert f["adaln_quant_gbs"] > 0 and f["rms_rope_q_k_gbs"] > 0
