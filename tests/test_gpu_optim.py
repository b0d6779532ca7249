"""GPU parity of the optimizer step: the gradient norm against the fp64
oracle, and the clipped AdamW update against the oracle's restatement of
update! (src/training/optimizer.jl:48-73, wan_runner.jl:213-221) bit for bit
-- moments, fp32 masters and the parameters' 16-bit copies -- over several
steps, across tensor lengths around the kernels' chunk size, parameter
types, weight-decay masks and pointers that rule out vector access."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

f32 = np.float32


@pytest.fixture(scope="module")
def torch():
    import torch as _t
    from reels_b200 import build
    build.build()
    return _t


def _bf16_round(x):
    return oracle.bf16_round(np.asarray(x, f32))


def _param_copy(w, dtype):
    if dtype == "bf16":
        return _bf16_round(w)
    if dtype == "f16":
        return w.astype(np.float16).astype(f32)
    return w


def _make(torch, sizes, dtypes, seed, offset=0):
    rng = np.random.default_rng(seed)
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
    params, grads = [], []
    for n, dt in zip(sizes, dtypes):
        w = (0.05 * rng.standard_normal(n)).astype(f32)
        g = rng.standard_normal(n).astype(f32) * f32(0.01)
        # `offset` elements in front shift the tensors off 16-byte alignment
        pbuf = torch.from_numpy(np.concatenate([np.zeros(offset, f32), w])).cuda().to(tdt[dt])
        gbuf = torch.from_numpy(np.concatenate([np.zeros(offset, f32), g])).cuda()
        params.append(pbuf[offset:])
        grads.append(gbuf[offset:])
    return params, grads


def _host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("offset", [0, 1])
def test_adamw_steps_match_oracle(torch, offset):
    from reels_b200 import check_device_status
    from reels_b200 import optim
    sizes = [1, 3, 8191, 8192, 8193, 100003, 0, 40000]
    dtypes = ["bf16", "f16", "f32", "bf16", "bf16", "f16", "bf16", "f32"]
    mask = [True, False, True, True, False, True, True, False]
    params, grads = _make(torch, sizes, dtypes, seed=5 + offset, offset=offset)
    opt = optim.AdamW(learning_rate=3e-4, weight_decay=0.02)
    state = optim.AdamWState(params)
    # the oracle's copy of the state
    om = [np.zeros(n, f32) for n in sizes]
    ov = [np.zeros(n, f32) for n in sizes]
    ow = [_host(p) for p in params]
    rng = np.random.default_rng(11)
    for step in range(1, 4):
        if step > 1:  # new gradients each step
            for g in grads:
                g.copy_(torch.from_numpy((0.01 * rng.standard_normal(g.numel())).astype(f32)))
        lr = optim.learning_rate(3e-4, "cosine", 1, step, 10)
        optim.update_(opt, state, params, grads, learning_rate=lr, weight_decay_mask=mask, grad_scale=0.5)
        c1, c2 = optim.bias_corrections(opt, step)
        for i, g in enumerate(grads):
            decay = f32(0.02) if mask[i] else f32(0.0)
            om[i], ov[i], ow[i] = oracle.adamw_update(_host(g), om[i], ov[i], ow[i], f32(lr), f32(0.9), f32(0.999),
                                                      f32(1e-8), decay, c1, c2, 0.5)
    check_device_status()
    for i, dt in enumerate(dtypes):
        assert np.array_equal(_host(state.m[i]), om[i]), (i, "m")
        assert np.array_equal(_host(state.v[i]), ov[i]), (i, "v")
        assert np.array_equal(_host(state.master[i]), ow[i]), (i, "master")
        assert np.array_equal(_host(params[i]), _param_copy(ow[i], dt)), (i, "param")


def test_grad_norm_and_clip(torch):
    from reels_b200 import check_device_status
    from reels_b200 import optim
    sizes = [5, 8192 * 3 + 7, 123457, 64]
    dtypes = ["bf16", "bf16", "f16", "f32"]
    params, grads = _make(torch, sizes, dtypes, seed=9)
    state = optim.AdamWState(params)
    ss = optim.grad_norm_sq(state, params, grads, grad_scale=0.25)
    ss2 = optim.grad_norm_sq(state, params, grads, grad_scale=0.25)
    ref = oracle.sumsq([_host(g) for g in grads], 0.25)
    assert abs(ss.item() - ref) <= 1e-6 * ref
    assert ss.item() == ss2.item()  # fixed summation order
    assert ss.item() == float(f32(ref))  # fp64 accumulation, rounded once: the oracle's fp32 value
    # clip: max_norm well below the norm
    w0 = [_host(p) for p in params]
    g0 = [_host(g) for g in grads]
    opt = optim.AdamW(learning_rate=1e-3, weight_decay=0.0)
    max_norm = 0.1 * float(np.sqrt(ref))
    sumsq = optim.update_(opt, state, params, grads, max_gradient_norm=max_norm, grad_scale=0.25)
    check_device_status()
    norm = np.sqrt(f32(sumsq.item()), dtype=f32)
    assert norm > max_norm
    clip = f32(f32(max_norm) / norm)
    c1, c2 = optim.bias_corrections(opt, 1)
    for i in range(len(sizes)):
        m, v, w = oracle.adamw_update(g0[i], np.zeros(sizes[i], f32), np.zeros(sizes[i], f32), w0[i], f32(1e-3),
                                      f32(0.9), f32(0.999), f32(1e-8), f32(0.0), c1, c2, 0.25, clip)
        assert np.array_equal(_host(state.m[i]), m), i
        assert np.array_equal(_host(state.master[i]), w), i


def test_unprepared_workspace_reports_an_error(torch):
    from reels_b200 import _native as nat
    L = nat.lib()
    ws = torch.zeros(L.reels_opt_workspace_bytes(4), dtype=torch.uint8, device="cuda")
    out = torch.zeros((), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert L.reels_grad_norm_sq(ws.data_ptr(), 1.0, out.data_ptr(), stream) == 0
    rc = L.reels_lowvram_check_device_status(stream)
    assert rc == nat.EDEVICE and "reels_opt_prepare" in L.reels_lowvram_last_error().decode()
    assert L.reels_lowvram_check_device_status(stream) == 0  # the status word was cleared


def test_reference_known_answers(torch):
    """test/unit/training.jl:87-127 on the GPU: exclusions give exactly 0.95
    and 1; an fp16 parameter moves, its fp32 master is kept, and the
    parameter equals the master rounded to fp16."""
    from reels_b200 import check_device_status
    from reels_b200 import optim
    params = [torch.ones(2, device="cuda"), torch.ones(2, device="cuda")]
    grads = [torch.zeros(2, device="cuda"), torch.zeros(2, device="cuda")]
    state = optim.AdamWState(params)
    mask = optim.weight_decay_mask(["blocks.0.attn.lora_A.weight", "blocks.0.attn.bias"], [r"bias$"])
    optim.update_(optim.AdamW(learning_rate=0.1, weight_decay=0.5), state, params, grads, weight_decay_mask=mask)
    check_device_status()
    assert params[0].cpu().tolist() == [float(f32(0.95))] * 2
    assert params[1].cpu().tolist() == [1.0, 1.0]
    p16 = torch.tensor([1.0, -2.0], device="cuda").to(torch.float16)
    st16 = optim.AdamWState([p16])
    assert st16.master[0].dtype == torch.float32 and st16.master[0].cpu().tolist() == [1.0, -2.0]
    optim.update_(optim.AdamW(learning_rate=1e-2, weight_decay=0.0), st16, [p16],
                  [torch.tensor([0.25, -0.5], device="cuda")])
    check_device_status()
    assert st16.step == 1
    assert st16.master[0].cpu().tolist() != [1.0, -2.0]
    assert torch.equal(p16, st16.master[0].to(torch.float16))
