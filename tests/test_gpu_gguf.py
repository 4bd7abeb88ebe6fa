"""GGUF bytes straight from the file to the kernels: tensors read by the GGUF
reader from a file (memory map) go to the GEMV / GEMM / dequant unchanged and
match the oracle on the same bytes."""
import numpy as np
import pytest
import torch

from planejaja_b200 import gguf as G
from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_K, Q5_K, Q6_K, Q8_0

pytestmark = pytest.mark.gpu


def test_gguf_tensors_through_the_kernels(tmp_path, oracle):
    from planejaja_b200.engine import CudaEngine
    eng = CudaEngine(0)
    specs = [("blk.0.ffn_gate.weight", Q4_K, 320, 2048), ("blk.0.ffn_down.weight", Q6_K, 256, 2304),
             ("blk.0.attn_q.weight", Q8_0, 96, 512), ("blk.0.attn_v.weight", Q5_K, 128, 1024)]
    recs = [(name, (k, n), t, Q.synthetic_weights(n, k, t, seed=n)) for name, t, n, k in specs]
    path = tmp_path / "m.gguf"
    G.write_minimal(str(path), recs, {"general.architecture": "llama"}, alignment=64)
    with G.open_gguf(str(path)) as f:
        for name, t, n, k in specs:
            assert f.tensors[name].matrix() == (n, k)
            raw = np.array(f.data(name))
            w = f.to_device(eng, name)
            x = Q.synthetic_activations(2, k, seed=k)
            y = eng.gemv(w, t, torch.from_numpy(x).to(eng.device), n, k).cpu().numpy()
            ref = oracle.quant_matmul(raw, t, x, n, k)
            rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
            assert np.max(np.abs(y - ref) / np.maximum(np.abs(ref), rms)) <= 1e-3, name
            d = eng.dequant(w, t, n * k).cpu().numpy()
            assert np.array_equal(d.view(np.uint32), oracle.dequant(raw, t).view(np.uint32)), name
    assert eng.device_status() == 0
