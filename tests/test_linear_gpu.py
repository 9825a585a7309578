"""tcgen05 projections (rt_linear) against an fp32 reference, and the fused epilogues
against the standalone stage kernels applied to the stored projection (bit-exact)."""

import pytest
import torch
import torch.nn.functional as F

from retree_b200 import _lib, kernels
from retree_b200.fused import FusedTarget
from retree_b200.target import build_target, qwen3_config
from tests.gpu_util import cuda

pytestmark = pytest.mark.gpu


def _data(m, n_out, k, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn((n_out, k), device=dev, generator=g) * k ** -0.5).to(torch.bfloat16)
    return x, w


def _check_store(x, w, y):
    ref = x.float() @ w.float().t()
    err = (y.float() - ref).abs()
    # bf16 output rounding (2^-8 relative) plus fp32 accumulation-order noise
    tol = ref.abs() * 2 ** -8 + 1e-3 * ref.abs().max()
    assert bool((err <= tol).all()), float((err - tol).max())


@pytest.mark.parametrize("m,n_out,k", [(1, 128, 64), (17, 2560, 4096), (17, 6144, 2560), (17, 2560, 9728),
                                       (33, 1024, 520), (65, 4096, 2560), (200, 768, 1024), (257, 2560, 2560),
                                       (300, 384, 256), (512, 256, 128)])
@torch.inference_mode()
def test_linear_store_matches_fp32_reference(m, n_out, k):
    dev = cuda()
    x, w = _data(m, n_out, k, m + n_out + k, dev)
    y = kernels.linear(x, w)
    kernels.check_device_status(dev)
    _check_store(x, w, y)
    # deterministic: split-K partials are summed in a fixed order
    assert torch.equal(kernels.linear(x, w), y)


@torch.inference_mode()
def test_linear_strided_input_and_output():
    dev = cuda()
    x, w = _data(40, 512, 1024, 3, dev)
    xs = torch.zeros((40, 1024 + 64), dtype=torch.bfloat16, device=dev)
    xs[:, :1024] = x
    out = torch.zeros((40, 512 + 128), dtype=torch.bfloat16, device=dev)
    kernels.linear(xs[:, :1024], w, out=out[:, :512])
    _check_store(x, w, out[:, :512])
    assert not out[:, 512:].any()


@pytest.mark.parametrize("m", [17, 65, 257])
@torch.inference_mode()
def test_linear_silu_mul_epilogue_equals_store_then_silu(m):
    dev = cuda()
    inter, k = 1024, 2560
    x, w = _data(m, 2 * inter, k, 7 + m, dev)
    y = kernels.linear(x, w)
    want = torch.empty((m, inter), dtype=torch.bfloat16, device=dev)
    kernels.silu_mul(y, want)
    got = kernels.linear(x, w, epilogue=_lib.RT_EPI_SILU_MUL)
    kernels.check_device_status(dev)
    assert torch.equal(got, want)
    assert torch.equal(want, F.silu(y[:, :inter]) * y[:, inter:])


@pytest.mark.parametrize("m,offset_dev", [(17, False), (41, True)])
@torch.inference_mode()
def test_linear_qkv_rope_epilogue_equals_store_then_rope(m, offset_dev):
    dev = cuda()
    cfg = qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=1, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=1000)
    model = build_target(cfg, device=dev, seed=2)
    attn = model.model.layers[0].self_attn
    with torch.no_grad():
        attn.q_norm.weight.copy_((1 + 0.2 * torch.randn(128, device=dev)).to(torch.bfloat16))
        attn.k_norm.weight.copy_((1 + 0.2 * torch.randn(128, device=dev)).to(torch.bfloat16))
    hq, hkv, k = 8, 2, 512
    x, w = _data(m, (hq + 2 * hkv) * 128, k, 11, dev)
    cos, sin = FusedTarget._rope_tables(model, 2048)
    pos = torch.randint(0, 2048, (m,), device=dev, generator=torch.Generator(device=dev).manual_seed(5))
    cap, off = 400, 123
    odev = torch.tensor([off - 3], dtype=torch.int64, device=dev) if offset_dev else None
    host_off = 3 if offset_dev else off

    def run(fused_epilogue):
        slab = torch.zeros((2, hkv, cap, 128), dtype=torch.bfloat16, device=dev)
        q = torch.empty((m, hq, 128), dtype=torch.bfloat16, device=dev)
        if fused_epilogue:
            kernels.linear(x, w, epilogue=_lib.RT_EPI_QKV_ROPE,
                           qkv=dict(num_q_heads=hq, num_kv_heads=hkv, q_norm=attn.q_norm.weight,
                                    k_norm=attn.k_norm.weight, eps=1e-6, cos=cos, sin=sin, positions=pos, q_out=q,
                                    k_cache=slab[0], v_cache=slab[1], offset=host_off, offset_dev=odev))
        else:
            y = kernels.linear(x, w)
            kernels.qk_norm_rope_append(y, hq, hkv, attn.q_norm.weight, attn.k_norm.weight, 1e-6, cos, sin, pos, q,
                                        slab[0], slab[1], offset=host_off, offset_dev=odev)
        kernels.check_device_status(dev)
        return q, slab

    q1, s1 = run(True)
    q2, s2 = run(False)
    assert torch.equal(q1, q2)
    assert torch.equal(s1, s2)
    assert s1[:, :, off: off + m].any() and not s1[:, :, :off].any() and not s1[:, :, off + m:].any()


@torch.inference_mode()
def test_linear_rejects_unsupported_shapes():
    dev = cuda()
    x, w = _data(8, 200, 64, 1, dev)   # n_out not a multiple of 128
    with pytest.raises(RuntimeError):
        kernels.linear(x, w)
    x, w = _data(513, 128, 64, 1, dev)  # more than 512 rows
    with pytest.raises(RuntimeError):
        kernels.linear(x, w)
