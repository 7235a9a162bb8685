"""bench.py's headline line: the contract's keys, one small entry per config, and short enough that
the whole line survives a 1500-character log tail (no GPU: a synthetic full record)."""
import json

import bench


def _full_record():
    sweep = [{"size": s, "mode": m, "ms_per_step": 1.234567, "tflops": 245.678901} for s in bench.SWEEP_SIZES
             for m in ("fp32x3", "tf32")]
    return {
        "metric": bench.METRIC, "value": 243.35952745583094, "unit": "TFLOP/s", "n_gpus": 8, "steps": 20,
        "warmup": 5, "ms_per_step": 4.518054580688476, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "tf32x3", "data": "synthetic N(0,1), fixed seeds",
        "config": {"workload": "config 4: square fp32 GEMM M=N=K=8192, fp32x3, M-row-block sharded over 8 GPU(s), "
                               "C gathered to GPU 0", "parallelism": "m-rows x8",
                   "l2": "inputs > L2 (256 MiB per operand), no flush", "math_mode": "fp32x3"},
        "roofline": {"bound": "tensor", "achieved": 262.89464420740944, "peak": 280.98333, "unit": "TFLOP/s",
                     "frac": 0.93562362, "traffic": 4890723328.0, "kernel": "gemm_tc_kernel", "kernel_ms": 4.18,
                     "peak_basis": "x" * 120, "frac_of_sustained_peak": 1.118066, "cublas_tf32_tflops": 733.2736739},
        "cpu_baseline": {"value": 1.0284341802911976, "unit": "TFLOP/s", "cores": 16, "kind": "reference",
                         "sample": "y" * 200},
        "clocks": {"sm_mhz": 1953.5, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 6},
        "e2e": {"value": 93.43723379976952, "unit": "TFLOP/s", "h2d_bytes_per_step": 536870912,
                "d2h_bytes_per_step": 268435456, "api": "z" * 100, "pcie_floor": {"ms_per_step": 2.0}},
        "gpu_launches": 60,
        "tf32_mode": {"value": 529.123456, "kernel_tflops": 548.987654, "roofline": {"frac": 0.6512345}},
        "sweep": {"results": sweep},
        "matmul512": {"value": 12.3456789},
        "cnn": {"value": 0.6789012},
        "attention": {"value": 0.4181234, "algorithmic_tflops_causal": 15.4712345},
        "transformer": {"value": 968765.4321, "ms_per_step": 33.8234567, "algorithmic_tflops": 91.4381727,
                        "e2e": {"value": 950123.456}},
        "cpu_baselines_other_configs": {"config1_matmul512_tflops": 0.6053642440260877,
                                        "config2_cnn_ms_per_step": 3.040396000002943,
                                        "config3_attention_ms_per_step": 41.9970869999986,
                                        "config5_transformer_tokens_per_s": 6230.324965353859},
        "gather_baseline": {"value": 410.123456},
    }


def test_headline_keeps_contract_keys_and_fits_a_short_tail():
    rec = _full_record()
    line = bench.headline(rec)
    text = bench.headline_text(rec)
    assert json.loads(text) == line
    assert len(text) <= 1450, len(text)
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "cpu_baseline", "e2e", "clocks",
              "gpu_launches"):
        assert k in line, k
    assert line["roofline"]["frac"] == 0.9356
    cfg = line["configs"]
    assert set(cfg) >= {"c1_tflops", "c2_ms", "c3", "c4_tf32", "c4_sweep_x3", "c5", "cpu"}
    assert len(cfg["c4_sweep_x3"]) == len(bench.SWEEP_SIZES)
