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
