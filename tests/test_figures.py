"""Every figure draws from a minimal payload into a well-formed SVG."""

import json
import xml.dom.minidom

from gpt2_harness_b200 import viz
from gpt2_harness_b200.perf.plots import fig_roofline, fig_step_breakdown
from gpt2_harness_b200.perf.roofline import MachinePeak, roofline_payload
from gpt2_harness_b200.utils.svg import nice_ticks


def _ok(p):
    xml.dom.minidom.parse(str(p))  # well-formed
    assert p.stat().st_size > 200


def test_nice_ticks():
    assert nice_ticks(0, 10) == [0, 2, 4, 6, 8, 10] or nice_ticks(0, 10) == [0, 2.5, 5, 7.5, 10]
    assert nice_ticks(1, 1000, log=True) == [1, 10, 100, 1000]


def test_perf_figures(tmp_path):
    pay = roofline_payload(MachinePeak("b200", "bf16", 1.4e15, 6.4e12, 218.0), batch=4, seq=256)
    _ok(fig_roofline(pay, tmp_path / "roof.svg"))
    _ok(fig_step_breakdown([{"label": "a", "categories": {"matmul": 0.6, "attention": 0.3}}], tmp_path / "s.svg"))


def test_science_figures_and_make_all(tmp_path):
    res = tmp_path / "results"
    res.mkdir()
    payloads = {
        "verification.json": {"layers": [{"max_abs": 1e-6}, {"max_abs": 3e-6}], "logit_tolerance": 1e-3},
        "induction.json": {"prefix_matching": [[0.1, 0.9], [0.2, 0.05]]},
        "ablations.json": {"rows": [{"label": "base", "verdict": "reference", "val_loss_mean": 3.0,
                                     "val_loss_std": 0.02},
                                    {"label": "relu", "verdict": "worse", "val_loss_mean": 3.1,
                                     "val_loss_std": 0.03}]},
        "kv_cache.json": {"rows": [{"arm": "cached", "prompt_len": 32, "ms_per_token": 3.6},
                                   {"arm": "native", "prompt_len": 32, "ms_per_token": 0.85},
                                   {"arm": "native", "prompt_len": 256, "ms_per_token": 0.81}],
                          "kv_cache": [{"seq_len": 1024, "batch_size": 1, "cache_mb": 37.7, "model_bytes": 5e8},
                                       {"seq_len": 2048, "batch_size": 1, "cache_mb": 75.4, "model_bytes": 5e8}]},
        "quantization.json": {"rows": [{"label": "fp32", "compression_ratio": 1.0, "ppl_mean": 20, "ppl_std": 1},
                                       {"label": "int4", "compression_ratio": 5.0, "ppl_mean": 22,
                                        "ppl_std": 1}]},
        "pruning.json": {"rows": [{"kind": "heads", "fraction_removed": 0.0, "val_loss": 3.0},
                                  {"kind": "heads", "fraction_removed": 0.1, "val_loss": 3.2}]},
        "distillation.json": {"runs": [{"label": "kd", "alpha": 0.5, "history": [{"step": 1, "val_loss": 5},
                                                                                 {"step": 2, "val_loss": 4}]}]},
        "pareto.json": {"points": [{"method": "int8", "size_mb": 150, "ppl": 21},
                                   {"method": "int4", "size_mb": 90, "ppl": 23}]},
        "pipeline_bubble.json": {"rows": [{"schedule": "1f1b", "micro_batches": m, "measured_bubble": 3 / (m + 3),
                                           "stages": 4} for m in (1, 2, 4, 8)]},
    }
    for k, v in payloads.items():
        (res / k).write_text(json.dumps(v))
    (res / "scaling.jsonl").write_text("\n".join(json.dumps({"n_gpus": n, "value": 7e5 * n}) for n in (1, 2, 4, 8)))
    out = viz.make_all(res, tmp_path / "fig")
    assert len(out) == len(payloads) + 2
    for p in out:
        _ok(p)
