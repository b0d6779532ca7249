"""Prequantised Int8 checkpoints on the GPU: the library's quantiser writes a
file whose loaded weight is bit-identical to quantising on load
(docs/src/training/low_vram.md:42-45 makes that claim for the reference), a
floating-point checkpoint converts on the GPU, and the loaded row-major
(in-contiguous) weight feeds the GEMMs directly."""
import numpy as np
import pytest

import lora_case as lc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as _t
    from reels_b200 import build
    build.build()
    return _t


def test_prequantised_file_is_bit_identical_to_on_load_quantisation(torch, tmp_path):
    from reels_b200 import checkpoint as ck
    from reels_b200 import quantize_frozen_matrix, weight_mul
    g = torch.Generator(device="cuda").manual_seed(5)
    w = torch.empty((640, 1024), device="cuda").normal_(0.0, 0.02, generator=g)  # [out, in], row-major
    on_load = quantize_frozen_matrix(w, torch.bfloat16)
    p = str(tmp_path / "w.safetensors")
    ck.write_quantized_checkpoint(p, {"blk.proj": on_load}, compute_dtype=torch.bfloat16)
    loaded = ck.load_quantized_linear(p, "blk.proj", 640, 1024, device="cuda", dtype=torch.bfloat16)
    assert torch.equal(loaded.values, on_load.values)
    assert torch.equal(loaded.scales.view(torch.int32), on_load.scales.view(torch.int32))
    x = torch.randn((300, 1024), device="cuda", generator=g).to(torch.bfloat16)
    y0 = weight_mul(on_load, x)
    y1 = weight_mul(loaded, x)
    assert torch.equal(y0, y1)
    # and the oracle agrees with the loaded (in-contiguous) weight
    q = loaded.values.cpu().numpy()
    s = loaded.scales.cpu().numpy()
    wdq = q.astype(np.float32) * s[:, None]
    ref = x.float().cpu().numpy() @ wdq.T
    assert lc.rel_l2(y1.float().cpu().numpy(), ref) <= lc.TOL


def test_quantize_checkpoint_on_gpu(torch, tmp_path):
    import oracle
    from reels_b200 import checkpoint as ck
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((96, 160)) * 0.02).astype(np.float32)
    w[5] = 0.0
    src, dst = str(tmp_path / "f.safetensors"), str(tmp_path / "q.safetensors")
    ck.write_safetensors(src, {"lin.weight": torch.from_numpy(w).to(torch.float16),
                               "lin.bias": torch.zeros(96, dtype=torch.float16)}, {"format": "float"})
    ck.quantize_checkpoint(src, dst, ["lin"], device="cuda", compute_dtype=torch.float16)
    h = ck.inspect_safetensors(dst)
    assert h.metadata["format"] == "float" and h.metadata["quantization"] == "int8-per-output-channel"
    assert "lin.bias" in h.tensors
    qm = ck.load_quantized_linear(dst, "lin", 96, 160, header=h)
    w16 = torch.from_numpy(w).to(torch.float16).float().numpy()
    q, s = oracle.quantize(w16, layout=oracle.LAYOUT_IN_CONTIGUOUS)
    assert np.array_equal(qm.values.numpy(), q)
    assert np.array_equal(qm.scales.numpy().view(np.uint32), s.view(np.uint32))
