"""CPU checks of the C ABI: the library loads, exports exactly what
include/*.h declares, and rejects bad arguments before touching a GPU
(status -1 plus a thread-local message, the convention of the reference's
deps/sentencepiece_bridge.cpp:10-17)."""
import ctypes
import glob
import os
import re

import pytest

from reels_b200 import _native as nat
from reels_b200 import build as native_build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(reels_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    native_build.build()
    return nat.lib()


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_functions()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    # and the binding table covers the header exactly
    assert sorted(nat.SIGNATURES) == declared


def test_abi_version(lib):
    assert lib.reels_lowvram_abi_version() == 1


def test_workspace_queries_need_no_gpu(lib):
    fw = lib.reels_q8lora_workspace_bytes(32760, 1536, 8960, 32, nat.BF16, nat.PASS_FORWARD)
    bw = lib.reels_q8lora_workspace_bytes(32760, 1536, 8960, 32, nat.BF16, nat.PASS_BACKWARD)
    assert fw > 0 and bw >= fw
    assert lib.reels_q8lora_workspace_bytes(-1, 1, 1, 0, nat.BF16, 0) == 0
    assert lib.reels_q8lora_saved_bytes(7, 3, nat.BF16) == 3 * 8 * 2   # tokens padded to 8
    assert lib.reels_q8lora_saved_bytes(32760, 32, nat.F16) == 32 * 32760 * 2
    assert lib.reels_q8lora_saved_bytes(5, 0, nat.BF16) == 0


def _err(lib):
    return lib.reels_lowvram_last_error().decode()


@pytest.mark.parametrize("bad", ["null_x", "neg_dim", "rank", "dtype", "layout"])
def test_forward_rejects_bad_arguments(lib, bad):
    p = ctypes.c_void_p(0x1000)  # never dereferenced: checks run first
    args = dict(x=p, q=p, s=p, layout=0, A=p, B=p, bias=None, M=4, K=16, N=16, r=2, alpha=2.0, dt=nat.BF16,
                y=p, saved=None, ws=None, wsn=0, stream=None)
    if bad == "null_x":
        args["x"] = None
    elif bad == "neg_dim":
        args["K"] = -3
    elif bad == "rank":
        args["r"] = 1000
    elif bad == "dtype":
        args["dt"] = 9
    elif bad == "layout":
        args["layout"] = 5
    rc = lib.reels_q8lora_forward(*args.values())
    assert rc == nat.EINVAL
    assert _err(lib) != ""


def test_backward_rejects_null_gradients(lib):
    p = ctypes.c_void_p(0x1000)
    rc = lib.reels_q8lora_backward(p, p, p, p, 0, p, p, None, 4, 16, 16, 2, 2.0, 1.0, nat.BF16, p, None, None,
                                   0, None, 0, None)
    assert rc == nat.EINVAL
    assert "dA" in _err(lib)


def test_empty_inputs_accept_null_token_buffers(lib):
    """M == 0 (and n == 0): the token-sized buffers may be NULL, the calls
    succeed without reading anything, and none of these touches a GPU."""
    p = ctypes.c_void_p(0x1000)
    assert lib.reels_q8lora_forward(None, p, p, 0, p, p, None, 0, 16, 16, 2, 2.0, nat.BF16, None, None, None, 0,
                                    None) == nat.OK
    assert lib.reels_q8lora_forward_act(None, p, p, 0, p, p, None, 0, 16, 16, 2, 2.0, nat.BF16, nat.ACT_GELU_TANH,
                                        None, None, None, None, 0, None) == nat.OK
    assert lib.reels_q8_weight_mul(None, p, p, 1, None, 0, 16, 16, nat.F16, None, None, 0, None) == nat.OK
    # dx only, no adapter: nothing to write
    assert lib.reels_q8_weight_transpose_mul(None, p, p, 0, 0, 16, 16, nat.BF16, None, None, 0, None) == nat.OK
    assert lib.reels_layernorm_modulate(None, 0, 16, 1, None, None, None, None, 1e-6, nat.BF16, None,
                                        None) == nat.OK
    assert lib.reels_gated_residual(None, None, None, 0, 16, 1, nat.BF16, None, None) == nat.OK
    assert lib.reels_dropout_mask(0, 0.5, 1, 0, None, None) == nat.OK
    # the weights themselves are never optional
    assert lib.reels_q8lora_forward(None, None, p, 0, p, p, None, 0, 16, 16, 2, 2.0, nat.BF16, None, None, None,
                                    0, None) == nat.EINVAL


def test_activation_entry_points_reject_bad_arguments(lib):
    p = ctypes.c_void_p(0x1000)
    q = ctypes.c_void_p(0x2000)
    fwd = lambda act, y, pre: lib.reels_q8lora_forward_act(p, p, p, 0, p, p, None, 4, 16, 16, 2, 2.0, nat.BF16,
                                                            act, y, pre, None, None, 0, None)
    assert fwd(7, p, q) == nat.EINVAL and "activation" in _err(lib)
    assert fwd(nat.ACT_GELU_TANH, p, p) == nat.EINVAL and "different" in _err(lib)
    bwd = lambda act, pre_x, dx: lib.reels_q8lora_backward_act(p, p, p, p, 0, p, p, None, 4, 16, 16, 2, 2.0, 1.0,
                                                                nat.BF16, act, pre_x, dx, p, p, 0, None, 0, None)
    assert bwd(3, q, p) == nat.EINVAL and "activation" in _err(lib)
    assert bwd(nat.ACT_GELU_TANH, None, p) == nat.EINVAL and "pre-activation" in _err(lib)
    assert bwd(nat.ACT_GELU_TANH, p, p) == nat.EINVAL and "different" in _err(lib)


def test_quantize_rejects_bad_arguments(lib):
    p = ctypes.c_void_p(0x1000)
    assert lib.reels_q8_quantize(None, nat.F32, 0, 4, 4, p, p, None) == nat.EINVAL
    assert lib.reels_q8_quantize(p, nat.F32, 0, 0, 4, p, p, None) == nat.EINVAL
    assert lib.reels_q8_materialize(p, p, 0, 4, 4, 7, p, None) == nat.EINVAL


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setenv("REELS_LOWVRAM_LIBRARY", str(tmp_path / "nope.so"))
    monkeypatch.setattr(nat, "_lib", None)
    with pytest.raises(RuntimeError, match="not found"):
        nat.lib()


def test_layer_api_mirrors():
    """lora_parameters (lora.jl:36-37) and frozen_weight_transfer's argument
    errors (quantization.jl:87-101), which need no GPU."""
    import torch
    from reels_b200 import LoRALinear, QuantizedMatrix, frozen_weight_transfer, lora_parameters
    qm = QuantizedMatrix(torch.zeros(6, 4, dtype=torch.int8), torch.ones(6), torch.float16)
    A = torch.zeros(2, 4, dtype=torch.float16)
    B = torch.zeros(6, 2, dtype=torch.float16)
    layer = LoRALinear(qm, None, A, B, 2.0)
    assert set(lora_parameters(layer)) == {"A", "B"}
    trained = LoRALinear(qm, torch.zeros(6, dtype=torch.float16), A, B, 2.0, train_bias=True)
    assert set(lora_parameters(trained)) == {"A", "B", "bias"}
    with pytest.raises(ValueError, match="none or int8"):
        frozen_weight_transfer("cuda", "fp16", quantization="int4")
    with pytest.raises(ValueError, match="requires device=cuda"):
        frozen_weight_transfer("cpu", "fp16", cpu_offload=True)
    with pytest.raises(ValueError, match="GPU path"):
        frozen_weight_transfer("cpu", "fp16", quantization="int8")
    t = frozen_weight_transfer("cpu", "fp32")
    w = torch.ones(3, 2, dtype=torch.float16)
    assert t(w).dtype == torch.float32


def test_quantized_matrix_getindex_rounds_the_scale_first():
    """getindex (quantization.jl:18-19) is T(q) * T(s): for Float16 the
    scale is rounded to Float16 before the product, so 127 * (1/3) gives
    42.3125, not the once-rounded 42.34375."""
    import torch
    from reels_b200 import QuantizedMatrix
    s = torch.tensor([1.0 / 3.0, 0.5], dtype=torch.float32)
    q = torch.tensor([[127, -3], [5, 0]], dtype=torch.int8)
    h = QuantizedMatrix(q, s, torch.float16)
    assert h[0, 0].item() == 42.3125 and h[0, 0].dtype == torch.float16
    assert h[1, 0].item() == 2.5 and h[1, 1].item() == 0.0
    f = QuantizedMatrix(q, s, torch.float32)
    assert f[0, 0].item() == float(torch.tensor(127.0) * s[0])


C_CONSUMER = r"""
#include <stdio.h>
#include <string.h>
#include "reels_lowvram.h"

int main(void) {
    int64_t info[7];
    int8_t q[16];
    float s[4];
    if (reels_lowvram_abi_version() != REELS_LOWVRAM_ABI_VERSION) return 1;
    if (reels_q8lora_workspace_bytes(32760, 1536, 8960, 32, REELS_BF16, REELS_PASS_BACKWARD) == 0) return 2;
    if (reels_q8lora_saved_bytes(7, 3, REELS_BF16) != 48) return 3;
    if (reels_q8_plan(32760, 1536, 8960, REELS_ACT_NONE, 148, info) != REELS_OK) return 4;
    if (info[3] < 1 || info[5] * info[6] < 1) return 5;
    if (reels_q8_quantize(NULL, REELS_F32, REELS_W_OUT_CONTIGUOUS, 4, 4, q, s, NULL) != REELS_EINVAL) return 6;
    if (strlen(reels_lowvram_last_error()) == 0) return 7;
    if (reels_opt_workspace_bytes(3) == 0) return 8;
    printf("ok %lld\n", (long long)info[0]);
    return 0;
}
"""


@pytest.mark.parametrize("compiler,std", [("gcc", "-std=c99"), ("g++", "-std=c++17")])
def test_header_serves_a_c_consumer(lib, tmp_path, compiler, std):
    """include/reels_lowvram.h compiles warning-free as C99 and C++ and links
    against the shared library, as a foreign-function binding sees it; the
    calls made need no GPU."""
    import shutil
    import subprocess
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} not installed")
    src = tmp_path / ("consumer.c" if compiler == "gcc" else "consumer.cpp")
    src.write_text(C_CONSUMER)
    exe = tmp_path / "consumer"
    libdir = os.path.dirname(nat.library_path())
    cmd = [compiler, std, "-pedantic", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           str(src), "-o", str(exe), "-L", libdir, "-lreels_lowvram", f"-Wl,-rpath,{libdir}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.startswith("ok"), (run.returncode, run.stdout, run.stderr)


def test_lora_fields_are_float32():
    """alpha and dropout are Float32 fields (lora.jl:6-7): the adapter scale
    alpha/rank is formed from the rounded alpha."""
    import torch
    from reels_b200 import LoRALinear, QuantizedMatrix
    qm = QuantizedMatrix(torch.zeros(6, 4, dtype=torch.int8), torch.ones(6), torch.float32)
    layer = LoRALinear(qm, None, torch.zeros(3, 4), torch.zeros(6, 3), 0.1, dropout=0.3)
    assert layer.alpha == float(torch.tensor(0.1, dtype=torch.float32)) and layer.alpha != 0.1
    assert layer.dropout == float(torch.tensor(0.3, dtype=torch.float32))
    with pytest.raises(ValueError, match="dropout"):
        LoRALinear(qm, None, torch.zeros(3, 4), torch.zeros(6, 3), 1.0, dropout=1.0)


def test_host_side_size_checks(monkeypatch):
    """Operands whose sizes disagree with the call are refused on the host
    before any launch (the kernels would read or write out of bounds); the
    device requirement is lifted here so the checks run without a GPU."""
    import torch
    from reels_b200 import (LoRALinear, QuantizedMatrix, gated_residual, gated_residual_backward, layernorm_modulate,
                            layernorm_modulate_backward, lora_backward, lora_forward, weight_mul)
    from reels_b200 import lowvram
    monkeypatch.setattr(lowvram, "_require_cuda", lambda *a: None)
    x = torch.zeros(8, 4, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="scale must have 8 entries"):
        layernorm_modulate(x, torch.zeros(1, 4, dtype=torch.bfloat16), None, tokens_per_sample=4)
    with pytest.raises(ValueError, match="LayerNorm weight"):
        layernorm_modulate(x, None, None, weight=torch.zeros(5, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="tokens_per_sample"):
        layernorm_modulate(x, None, None, tokens_per_sample=0)
    with pytest.raises(ValueError, match="dout must have the shape"):
        layernorm_modulate_backward(x, torch.zeros(8, 5, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="gate must have 8 entries"):
        gated_residual(x, x, torch.zeros(1, 4, dtype=torch.bfloat16), tokens_per_sample=4)
    with pytest.raises(ValueError, match="out must be a contiguous"):
        gated_residual(x, x, torch.zeros(1, 4, dtype=torch.bfloat16), out=torch.zeros(4, 8, dtype=torch.bfloat16).t())
    with pytest.raises(ValueError, match="y and dout"):
        gated_residual_backward(x, x.float(), torch.zeros(1, 4))
    qm = QuantizedMatrix(torch.zeros(6, 4, dtype=torch.int8), torch.ones(6), torch.bfloat16)
    with pytest.raises(ValueError, match="bias must have 6 entries"):
        weight_mul(qm, x, torch.zeros(5, dtype=torch.bfloat16))
    layer = LoRALinear(qm, torch.zeros(7, dtype=torch.bfloat16), torch.zeros(2, 4, dtype=torch.bfloat16),
                       torch.zeros(6, 2, dtype=torch.bfloat16), 2.0)
    with pytest.raises(ValueError, match="bias must have 6 entries"):
        lora_forward(layer, x)
    layer.bias = None
    dy = torch.zeros(8, 6, dtype=torch.bfloat16)
    good_A, good_B = torch.zeros(4, 2).t(), torch.zeros(2, 6).t()
    with pytest.raises(ValueError, match="shapes of A"):
        lora_backward(layer, x, dy, dA_acc=torch.zeros(4, 3).t(), dB_acc=good_B)
    with pytest.raises(ValueError, match="fp32"):
        lora_backward(layer, x, dy, dA_acc=good_A.bfloat16(), dB_acc=good_B)
    with pytest.raises(ValueError, match="column-major"):
        lora_backward(layer, x, dy, dA_acc=torch.zeros(2, 4), dB_acc=good_B)
    with pytest.raises(ValueError, match="together"):
        lora_backward(layer, x, dy, dA_acc=good_A)


def test_empty_batches_through_the_layer_api(monkeypatch):
    """The Python mirror with no tokens: shapes and the early returns of the
    parameter-gradient pullbacks, on CPU (the native calls made here return
    before any device work when M == 0)."""
    import torch
    from reels_b200 import (LoRALinear, QuantizedMatrix, gated_residual, gated_residual_backward, layernorm_modulate,
                            layernorm_modulate_backward, lora_forward)
    from reels_b200 import lowvram
    monkeypatch.setattr(lowvram, "_require_cuda", lambda *a: None)
    monkeypatch.setattr(lowvram, "_stream", lambda d: 0)
    monkeypatch.setattr(lowvram, "_workspace", lambda *a: (None, 0))
    qm = QuantizedMatrix(torch.zeros(6, 4, dtype=torch.int8).t().contiguous().t(), torch.ones(6), torch.bfloat16)
    layer = LoRALinear(qm, None, torch.zeros(2, 4, dtype=torch.bfloat16), torch.zeros(6, 2, dtype=torch.bfloat16), 2.0)
    x = torch.empty((3, 0, 4), dtype=torch.bfloat16)
    assert tuple(lora_forward(layer, x).shape) == (3, 0, 6)
    scale = torch.zeros((2, 4), dtype=torch.bfloat16)
    assert tuple(layernorm_modulate(x, scale, scale, tokens_per_sample=5).shape) == (3, 0, 4)
    dx, ds, dh = layernorm_modulate_backward(x, x, scale, param_grads=True)
    assert tuple(dx.shape) == (3, 0, 4) and tuple(ds.shape) == (2, 4) and not ds.any() and not dh.any()
    gate = torch.ones((2, 4), dtype=torch.bfloat16)
    assert tuple(gated_residual(x, x, gate).shape) == (3, 0, 4)
    dyr, dg = gated_residual_backward(x, x, gate)
    assert tuple(dyr.shape) == (3, 0, 4) and tuple(dg.shape) == (2, 4) and not dg.any()
