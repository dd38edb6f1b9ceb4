"""Fused bf16 RMSNorm (``rms_norm`` / C-ABI ``dspark_rms_norm``) vs transformers'
``Qwen3RMSNorm`` run on the same GPU (models/qwen3/modeling_qwen3.py:62-66), the
norm of the target's decoder layers and final norm.

Every step rounds as torch's sequence does; only the association of the float sum
of squares differs, so an output may move by one bf16 ulp where the variance lands
next to a rounding boundary. The gate: at least 99.9% of outputs bit-identical and
none further than one bf16 ulp.
"""
import numpy as np
import pytest
import torch

from gpu_util import dev, status_clean

pytestmark = pytest.mark.gpu


def hf_norm(weight, eps):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    m = Qwen3RMSNorm(weight.numel(), eps=eps).to(dev(), torch.bfloat16)
    with torch.no_grad():
        m.weight.copy_(weight)
    return m


def ulp_distance(a, b):
    """Distance in bf16 steps between same-shaped bf16 tensors (ordered bit patterns)."""
    def key(t):
        bits = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(bits < 0, -(bits & 0x7fff), bits)
    return (key(a) - key(b)).abs()


def inputs(seed, rows, hidden, scale=1.0):
    g = np.random.Generator(np.random.PCG64(seed))
    x = torch.from_numpy(g.standard_normal((rows, hidden)).astype(np.float32) * scale).to(dev(), torch.bfloat16)
    w = torch.from_numpy(1.0 + 0.1 * g.standard_normal(hidden).astype(np.float32)).to(dev(), torch.bfloat16)
    return x, w


@pytest.mark.parametrize('rows,hidden,scale', [(1, 128, 1.0), (7, 256, 3.0), (256, 1024, 1.0), (33, 2560, 0.05),
                                               (5, 4096, 1.0), (300, 5120, 20.0), (4099, 1024, 1.0)])
def test_rms_norm_matches_transformers(pkg, rows, hidden, scale):
    x, w = inputs(rows * 7 + hidden, rows, hidden, scale)
    eps = 1e-6
    with torch.no_grad():
        ref = hf_norm(w, eps)(x)
    got = pkg.rms_norm(x, w, eps)
    torch.cuda.synchronize()
    assert got.shape == ref.shape and got.dtype == torch.bfloat16
    d = ulp_distance(got, ref)
    assert int(d.max()) <= 1
    assert float((d == 0).float().mean()) >= 0.999
    status_clean(pkg)


def test_rms_norm_packed_row_shape_strides_and_edges(pkg):
    x, w = inputs(5, 64, 1024)
    # the decoder layer's [1, n, hidden] input keeps its shape
    got = pkg.rms_norm(x[None], w, 1e-6)
    assert got.shape == (1, 64, 1024)
    assert torch.equal(got[0], pkg.rms_norm(x, w, 1e-6))
    # rows taken from a wider buffer (row stride 1088) give the same values as packed rows
    wide = torch.zeros((64, 1088), dtype=torch.bfloat16, device=dev())
    wide[:, 32:32 + 1024] = x
    assert torch.equal(pkg.rms_norm(wide[:, 32:32 + 1024], w, 1e-6), got[0])
    # zeros stay zeros (rsqrt(eps) times 0); squares that overflow float give zeros as in torch
    edge = x.clone()
    edge[0] = 0
    edge[1] = 1e30
    ref = hf_norm(w, 1e-6)(edge)
    mine = pkg.rms_norm(edge, w, 1e-6)
    assert torch.equal(mine[:2], ref[:2]) and not mine[:2].any()
    # no rows: nothing launched, empty result
    empty = pkg.rms_norm(x[:0], w, 1e-6)
    assert empty.shape == (0, 1024)
    with pytest.raises(ValueError):
        pkg.rms_norm(x.float(), w, 1e-6)
    with pytest.raises(ValueError):
        pkg.rms_norm(x[:, :1020], w[:1020], 1e-6)
    status_clean(pkg)


def test_bf16_target_runs_its_norms_fused_and_restores_them(pkg):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    import inputs as I
    cfg = Qwen3Config(**I.TINY_TARGET)
    model = Qwen3ForCausalLM(cfg).eval().to(dev(), torch.bfloat16)
    norms = [m for layer in model.model.layers for m in (layer.input_layernorm, layer.post_attention_layernorm)]
    norms.append(model.model.norm)
    target = pkg.B200Qwen3Target(model, (), slots=1, context_capacity=64, max_query_tokens=64)
    assert all('forward' in vars(m) for m in norms)
    target.add_request('r')
    before = pkg.launch_count()
    target.prefill({'r': torch.arange(16, device=dev())[None]})
    torch.cuda.synchronize()
    # per layer two norms plus the fused verify launch(es); the final norm once
    assert pkg.launch_count() - before >= len(norms) + cfg.num_hidden_layers
    target.close()
    assert not any('forward' in vars(m) for m in norms)
    status_clean(pkg)


def integer_rows(seed, rows, width, bound):
    """bf16 rows of small integers: every partial sum of squares is an exact float, so
    the sum no longer depends on its association and results must be bit-identical."""
    g = np.random.Generator(np.random.PCG64(seed))
    return torch.from_numpy(g.integers(-bound, bound + 1, (rows, width)).astype(np.float32)).to(dev(),
                                                                                              torch.bfloat16)


def test_rms_norm_bit_exact_when_the_sum_is_exact(pkg):
    x = integer_rows(3, 300, 1024, 8)
    _, w = inputs(4, 1, 1024)
    with torch.no_grad():
        ref = hf_norm(w, 1e-6)(x)
    assert torch.equal(pkg.rms_norm(x, w, 1e-6), ref)
    status_clean(pkg)


def rope_reference(x, heads, weight, eps, cos, sin):
    """The draft's torch path: Qwen3RMSNorm over each head, then rotate-half RoPE."""
    from importlib import import_module
    rotate = import_module('qwen3-dspark_b200.draft').rotate_half_rope
    n = x.shape[0]
    with torch.no_grad():
        y = hf_norm(weight, eps)(x.view(1, n, heads, 128)).transpose(1, 2)
        return rotate(y, cos, sin)[0].transpose(0, 1).contiguous()


def rope_tables(n, seed):
    import inputs as I
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    rot = Qwen3RotaryEmbedding(Qwen3Config(**I.TINY_TARGET)).to(dev())
    g = np.random.Generator(np.random.PCG64(seed))
    pos = torch.from_numpy(g.integers(0, 40000, n)).to(dev())
    return rot(torch.zeros(1, dtype=torch.bfloat16, device=dev()), pos[None])


@pytest.mark.parametrize('exact', [False, True])
def test_qk_norm_rope_matches_the_draft_torch_path(pkg, exact):
    n, hq, hkv = 224, 16, 8
    if exact:
        q, k = integer_rows(5, n, hq * 128, 6), integer_rows(6, n, hkv * 128, 6)
    else:
        q, _ = inputs(5, n, hq * 128, 2.0)
        k, _ = inputs(6, n, hkv * 128, 0.3)
    _, qw = inputs(7, 1, 128)
    _, kw = inputs(8, 1, 128)
    cos, sin = rope_tables(n, 9)
    assert cos.dtype == torch.bfloat16 and cos.shape == (1, n, 128)
    got_q, got_k = pkg.qk_norm_rope(q, k, qw, kw, 1e-6, 1e-6, cos[0], sin[0], hq, hkv)
    ref_q = rope_reference(q, hq, qw, 1e-6, cos, sin)
    ref_k = rope_reference(k, hkv, kw, 1e-6, cos, sin)
    for got, ref in ((got_q, ref_q), (got_k, ref_k)):
        assert got.shape == ref.shape
        if exact:
            assert torch.equal(got, ref)
        else:
            diff = (got.float() - ref.float()).abs()
            assert float(diff.max()) <= 2e-2
            assert float((diff == 0).float().mean()) >= 0.999
    status_clean(pkg)


def test_qk_norm_rope_row_strides_and_refusals(pkg):
    n = 9
    q, _ = inputs(10, n, 2 * 128 + 64)                   # rows of a wider buffer: stride 320
    k, _ = inputs(11, n, 128)
    _, w = inputs(12, 1, 128)
    cos, sin = rope_tables(n, 13)
    got_q, got_k = pkg.qk_norm_rope(q[:, :256], k, w, w, 1e-6, 1e-6, cos[0], sin[0], 2, 1)
    want_q, want_k = pkg.qk_norm_rope(q[:, :256].contiguous(), k, w, w, 1e-6, 1e-6, cos[0], sin[0], 2, 1)
    assert torch.equal(got_q, want_q) and torch.equal(got_k, want_k)
    empty_q, empty_k = pkg.qk_norm_rope(q[:0, :256], k[:0], w, w, 1e-6, 1e-6, cos[0, :0], sin[0, :0], 2, 1)
    assert empty_q.shape == (0, 2, 128) and empty_k.shape == (0, 1, 128)
    with pytest.raises(ValueError):
        pkg.qk_norm_rope(q[:, :256].float(), k, w, w, 1e-6, 1e-6, cos[0], sin[0], 2, 1)
    with pytest.raises(ValueError):
        pkg.qk_norm_rope(q[:, :256], k, w, w, 1e-6, 1e-6, cos[0], sin[0], 3, 1)
    status_clean(pkg)


def test_silu_mul_matches_torch_silu_times_up(pkg):
    g = np.random.Generator(np.random.PCG64(21))
    gu = torch.from_numpy(g.standard_normal((257, 2 * 3072)).astype(np.float32) * 3).to(dev(), torch.bfloat16)
    gu[0, :16] = torch.tensor([0, -0.0, 1e-30, -1e-30, 88, -88, 100, -100, 1e4, -1e4, 3e38, -3e38,
                               float('inf'), float('-inf'), 0.5, -0.5])
    got = pkg.silu_mul(gu, 3072)
    with torch.no_grad():
        ref = torch.nn.functional.silu(gu[:, :3072]) * gu[:, 3072:]
    same = (got.view(torch.int16) == ref.view(torch.int16)) | (torch.isnan(got) & torch.isnan(ref))
    finite = torch.isfinite(ref) & torch.isfinite(got)
    assert float(same.float().mean()) >= 0.999
    assert int(ulp_distance(torch.where(finite, got, 0), torch.where(finite, ref, 0)).max()) <= 1
    assert torch.equal(torch.isnan(got), torch.isnan(ref))
    # rows of a wider buffer and the empty case
    wide = torch.zeros((257, 2 * 3072 + 64), dtype=torch.bfloat16, device=dev())
    wide[:, :2 * 3072] = gu
    assert torch.equal(pkg.silu_mul(wide[:, :2 * 3072], 3072).view(torch.int16), got.view(torch.int16))
    assert pkg.silu_mul(gu[:0], 3072).shape == (0, 3072)
    with pytest.raises(ValueError):
        pkg.silu_mul(gu, 3000)
    status_clean(pkg)


def test_bf16_target_mlp_runs_merged_and_matches_transformers(pkg):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    import inputs as I
    cfg = Qwen3Config(**I.TINY_TARGET)
    model = Qwen3ForCausalLM(cfg).eval().to(dev(), torch.bfloat16)
    mlp = model.model.layers[1].mlp
    x, _ = inputs(31, 40, cfg.hidden_size)
    with torch.no_grad():
        ref = mlp(x[None])
        gate_before = mlp.gate_proj.weight.clone()
    target = pkg.B200Qwen3Target(model, (), slots=1, context_capacity=64, max_query_tokens=64)
    assert 'forward' in vars(mlp)
    assert torch.equal(mlp.gate_proj.weight, gate_before)              # views of the merged buffer, same values
    assert mlp.up_proj.weight.data_ptr() == mlp.gate_proj.weight.data_ptr() + mlp.gate_proj.weight.numel() * 2
    with torch.no_grad():
        got = mlp(x[None])
    err = (got.float() - ref.float()).abs().max().item()
    assert err <= 0.02 * ref.float().abs().max().item() + 1e-3, err
    target.close()
    assert 'forward' not in vars(mlp)
    status_clean(pkg)


@pytest.mark.parametrize('exact', [False, True])
def test_add_rms_norm_matches_torch_add_then_transformers_norm(pkg, exact):
    if exact:
        x, d = integer_rows(40, 300, 1024, 4), integer_rows(41, 300, 1024, 4)
    else:
        x, _ = inputs(40, 300, 1024, 4.0)
        d, _ = inputs(41, 300, 1024, 0.5)
    _, w = inputs(42, 1, 1024)
    with torch.no_grad():
        s = x + d
        ref = hf_norm(w, 1e-6)(s)
    got_s, got = pkg.add_rms_norm(x, d, w, 1e-6)
    assert torch.equal(got_s, s)                      # the residual sum is torch's bf16 add
    if exact:
        assert torch.equal(got, ref)
    else:
        dist = ulp_distance(got, ref)
        assert int(dist.max()) <= 1 and float((dist == 0).float().mean()) >= 0.999
    empty_s, empty = pkg.add_rms_norm(x[:0], d[:0], w, 1e-6)
    assert empty_s.shape == empty.shape == (0, 1024)
    status_clean(pkg)
