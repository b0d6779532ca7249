"""GPU: every C-ABI entry point runs on the device that owns its buffers and
returns with the caller's current device unchanged (include/reels_lowvram.h,
threading contract).  A caller with device 0 current passes device-1 buffers;
afterwards device 0 is still current.  Needs two GPUs (skipped otherwise),
except the one-GPU case that the current device stays put."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    from reels_b200 import build
    build.build()
    return torch


def _layer(torch, dev, N=256, K=512, r=16):
    from reels_b200 import LoRALinear, quantize_frozen_matrix
    g = np.random.default_rng(3)
    W = torch.from_numpy((0.02 * g.standard_normal((N, K))).astype(np.float32)).to(dev)
    qm = quantize_frozen_matrix(W, torch.bfloat16)
    A = torch.from_numpy((g.standard_normal((r, K)) / np.sqrt(K)).astype(np.float32)).to(dev).to(torch.bfloat16)
    B = torch.from_numpy((0.01 * g.standard_normal((N, r))).astype(np.float32)).to(dev).to(torch.bfloat16)
    return LoRALinear(qm, None, A, B, float(r))


def _call_raw(torch, layer, x, dy):
    """Forward, backward and the quantiser through the C ABI directly, on the
    buffers' device's default stream, with no torch device guard around."""
    from reels_b200 import _native as nat
    L = nat.lib()
    N, K = layer.weight.shape
    r = layer.rank
    M = x.shape[0]
    dev = x.device
    A_mem = layer.A.t().contiguous()
    B_mem = layer.B.t().contiguous()
    y = torch.empty((M, N), dtype=x.dtype, device=dev)
    nws = L.reels_q8lora_workspace_bytes(M, K, N, r, nat.BF16, nat.PASS_BACKWARD)
    ws = torch.empty(nws + 256, dtype=torch.uint8, device=dev)
    wp = ws.data_ptr() + (-ws.data_ptr()) % 256
    vals = layer.weight.values
    wptr = vals.data_ptr()
    rc = L.reels_q8lora_forward(x.data_ptr(), wptr, layer.weight.scales.data_ptr(), layer.weight.layout,
                                A_mem.data_ptr(), B_mem.data_ptr(), None, M, K, N, r, layer.alpha, nat.BF16,
                                y.data_ptr(), None, wp, nws, None)
    nat.check("forward", rc)
    dx = torch.empty((M, K), dtype=x.dtype, device=dev)
    dA = torch.empty((K, r), dtype=torch.float32, device=dev)
    dB = torch.empty((r, N), dtype=torch.float32, device=dev)
    rc = L.reels_q8lora_backward(x.data_ptr(), dy.data_ptr(), wptr, layer.weight.scales.data_ptr(),
                                 layer.weight.layout, A_mem.data_ptr(), B_mem.data_ptr(), None, M, K, N, r,
                                 layer.alpha, 1.0, nat.BF16, dx.data_ptr(), dA.data_ptr(), dB.data_ptr(), 0, wp, nws,
                                 None)
    nat.check("backward", rc)
    w = torch.ones((N, K), dtype=torch.float32, device=dev)
    q = torch.empty((N, K), dtype=torch.int8, device=dev)
    s = torch.empty((N,), dtype=torch.float32, device=dev)
    rc = L.reels_q8_quantize(w.data_ptr(), nat.F32, nat.W_IN_CONTIGUOUS, N, K, q.data_ptr(), s.data_ptr(), None)
    nat.check("quantize", rc)
    return y, dx


def test_current_device_kept_one_gpu(torch_cuda):
    torch = torch_cuda
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    layer = _layer(torch, dev)
    x = torch.randn((128, 512), device=dev).to(torch.bfloat16)
    dy = torch.randn((128, 256), device=dev).to(torch.bfloat16)
    _call_raw(torch, layer, x, dy)
    assert torch.cuda.current_device() == 0


def test_caller_device_restored_two_gpus(torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from reels_b200 import lora_backward, lora_forward
    d1 = torch.device("cuda", 1)
    layer = _layer(torch, d1)
    x = torch.randn((128, 512), device=d1).to(torch.bfloat16)
    dy = torch.randn((128, 256), device=d1).to(torch.bfloat16)
    torch.cuda.set_device(1)
    y_ref = lora_forward(layer, x)
    dx_ref = lora_backward(layer, x, dy).dx
    torch.cuda.synchronize(d1)
    torch.cuda.set_device(0)
    y, dx = _call_raw(torch, layer, x, dy)
    assert torch.cuda.current_device() == 0       # the caller's device is back
    torch.cuda.synchronize(d1)
    assert torch.equal(y, y_ref) and torch.equal(dx, dx_ref)
