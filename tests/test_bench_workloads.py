"""The benchmark's workload tables: shapes, activation wiring and byte counts (CPU)."""
import pytest

import bench
from planejaja_b200.formats import fmt

MB = 1e6


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_workload_wiring(name):
    w = bench.WORKLOADS[name]
    names = [n for n, _, _, _ in w["spec"]]
    grouped = [n for _, g in w["groups"] for n in g]
    assert sorted(grouped) == sorted(names), "every projection in exactly one fused launch"
    for a, g in w["groups"]:
        for nm in g:
            assert w["act_of"][nm] == a
    for nm, n, k, t in w["spec"]:
        assert k == w["act_k"][w["act_of"][nm]], nm
        assert k % 256 == 0, "the fused decode kernel walks K in 256-weight pieces"
        assert fmt(t).row_bytes(k) % 16 == 0, "rows are copied with 16-byte-aligned bulk copies"


@pytest.mark.parametrize("name,layer_mb", [("l3-8b", 138.90), ("l2-7b", 113.84), ("l2-70b-ffn", 3 * 132.12)])
def test_layer_weight_bytes(name, layer_mb):
    # Llama-3-8B Q4_K_M: 138.90 MB per layer; Llama-2-7B Q4_0: 113.84 MB;
    # Llama-2-70B FFN Q4_K: 3 x 132.12 MB
    w = bench.WORKLOADS[name]
    total = sum(fmt(t).tensor_bytes(n, k) for _, n, k, t in w["spec"])
    assert abs(total / MB - layer_mb) < 0.01


def test_select_workload_rebinds():
    try:
        bench.select_workload("l2-7b", 1)
        assert bench.METRIC == "decode GEMV HBM GB/s (Llama-2-7B Q4_0, M=1)"
        assert {t for _, _, _, t in bench.LAYER_SPEC} == {2}
        wb, xb, yb = bench.layer_bytes_total()
        assert xb == 4 * (6 * 4096 + 11008) and yb == 4 * (5 * 4096 + 2 * 11008)
    finally:
        bench.select_workload("l3-8b", 1)


def test_reference_arm_json_line():
    """`bench.py --impl reference` runs the oracle on the host and prints one
    JSON line with the GPU arm's metric, a cpu_baseline and an e2e entry."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3", "--ref-frac", "0.005"], capture_output=True, text=True, timeout=600,
                         cwd=root, env={**os.environ, "WORLD_SIZE": "1", "RANK": "0"})
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "decode GEMV HBM GB/s (Llama-3-8B Q4_K_M, M=1)"
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["steps"] == 1 and line["warmup"] == 3
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_row_shards_are_slices_of_the_whole_matrix():
    """Each rank quantizes only its rows; the bytes equal that slice of the whole matrix."""
    import numpy as np
    from planejaja_b200 import quantize as Q
    n, k = 6000, 512
    whole = Q.synthetic_weights(n, k, 12, seed=5)
    rb = fmt(12).row_bytes(k)
    for world in (2, 4, 8):
        parts = [Q.synthetic_weights(n, k, 12, seed=5, rows=(r * n // world, (r + 1) * n // world))
                 for r in range(world)]
        assert np.array_equal(np.concatenate(parts), whole)
        assert parts[1].size == (n // world) * rb


def test_single_thread_reference_loop_on_a_small_layer():
    """The reference-order CPU leg (dequant, transpose, stride-N cpu_matmul_f32) on a tiny layer."""
    try:
        bench.select_workload("l3-8b", 1)
        spec = [("q", 64, 512, 12), ("v", 32, 512, 14)]
        saved = bench.LAYER_SPEC, bench.ACT_OF
        bench.LAYER_SPEC, bench.ACT_OF = spec, {"q": 0, "v": 0}
        from planejaja_b200 import quantize as Q
        layer = {nm: Q.synthetic_weights(n, k, t, seed=1) for nm, n, k, t in spec}
        acts = [Q.synthetic_activations(1, 512, seed=2).reshape(-1)]
        rec = bench.cpu_leg_reference_loop(layer, acts)
        assert rec["cores"] == 1 and rec["value"] > 0 and rec["matmul_s"] >= 0
        assert "stride-N" in rec["loop"]
    finally:
        bench.LAYER_SPEC, bench.ACT_OF = saved
        bench.select_workload("l3-8b", 1)
