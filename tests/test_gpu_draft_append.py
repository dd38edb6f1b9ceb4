"""Fused draft-context append (``dspark_draft_append``) against the reference's
formula (PackedDraft.append_committed + DraftAttention.project_kv,
packed_draft.py:129-168, model.py:41-45) run with torch ops in the same dtype.

* every layer's pool K (k_norm + RoPE of k_proj) and V (v_proj) of appended rows
  match the torch formula within the bf16 gate, at the 0.6B draft geometry
  (hidden 1024, five layers) and with ragged requests;
* the fixed-shape verified-chunk append writes the committed rows only: every other
  pool row except the trash row is bit-identical to before;
* the captured append replays bit-identically to the eager one;
* a destination outside the pool is skipped and reported in the device status.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, dev, status_clean

pytestmark = pytest.mark.gpu

FEATURES = 2


def build_draft(pkg, hidden=1024, layers=5, seed=0):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(seed)
    cfg = Qwen3Config(vocab_size=1024, hidden_size=hidden, intermediate_size=2 * hidden, num_hidden_layers=4,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                      rms_norm_eps=1e-6, tie_word_embeddings=False,
                      rope_parameters={'rope_type': 'default', 'rope_theta': 1e6})
    with torch.device(dev()), torch.no_grad():
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
        spec = pkg.DraftSpec(layer_ids=(1, 2), num_layers=layers, block_size=7, markov_rank=64, mask_token_id=1000)
        draft = pkg.DSparkDraftModel(model, spec).to(torch.bfloat16).eval()
        for layer in draft.layers:      # non-trivial k_norm weights
            layer.attention.k_norm.weight.copy_(1 + 0.1 * torch.randn_like(layer.attention.k_norm.weight))
    return draft


def pools(pd):
    return [t.clone() for t in pd.pool_k], [t.clone() for t in pd.pool_v]


def features(g, n, hidden):
    return torch.from_numpy(g.standard_normal((1, n, FEATURES * hidden)).astype(np.float32)).to(dev(),
                                                                                                torch.bfloat16)


# (1024, 5) with the 1131-row first append runs the 2-SM kernel (tiles of 256 rows x 2
# heads over CTA pairs; the last pair tile's second CTA reads past the input rows), the
# others the single-CTA kernels with one or two heads per tile.
@pytest.mark.parametrize('hidden,layers,lens,capacity', [
    (1024, 5, [(1, 37), (300, 5), (129, 128), (2, 0)], 700),
    (256, 2, [(1, 37), (300, 5), (129, 128), (2, 0)], 700),
    (1024, 5, [(700, 37), (300, 5), (129, 128), (2, 0)], 1000),
])
def test_fused_append_matches_torch_formula(pkg, hidden, layers, lens, capacity):
    draft = build_draft(pkg, hidden, layers)
    fused = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=capacity)
    plain = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=capacity)
    assert fused._fused_append_ready()
    plain._fused_append_ready = lambda: False
    g = np.random.Generator(np.random.PCG64(5))
    for i in range(4):
        for pd in (fused, plain):
            pd.add_request(f'r{i}')
    for step in range(2):                                   # second append lands after the first
        chunks = {f'r{i}': features(g, lens[i][step], hidden) for i in range(4) if lens[i][step]}
        fused.append_committed(chunks)
        plain.append_committed(chunks)
        assert fused.lengths == plain.lengths
        assert fused.last_projection_work['kv_projection_calls'] == 1
    for i in range(4):
        for (fk, fv), (pk, pv) in zip(fused.request_kv(f'r{i}'), plain.request_kv(f'r{i}')):
            assert_bf16_close(fk, pk.float().cpu().numpy())
            assert_bf16_close(fv, pv.float().cpu().numpy())
    status_clean(pkg)


def test_verified_append_writes_committed_rows_only(pkg):
    draft = build_draft(pkg)
    pd = pkg.B200PackedDraft(draft, max_requests=3, context_capacity=400)
    twin = pkg.B200PackedDraft(draft, max_requests=3, context_capacity=400)
    g = np.random.Generator(np.random.PCG64(6))
    reqs = ('a', 'b', 'c')
    for pdx in (pd, twin):
        for r in reqs:
            pdx.add_request(r)
    ctx = {r: features(g, n, 1024) for r, n in zip(reqs, (50, 3, 200))}
    pd.append_committed(ctx)
    twin.append_committed(ctx)
    q = 8
    feat = features(g, 3 * q, 1024)
    counts = [0, 3, 8]
    before_k, before_v = pools(pd)
    pd.append_verified(feat, reqs, counts)
    twin.append_committed({r: feat[:, i * q:i * q + c] for i, (r, c) in enumerate(zip(reqs, counts)) if c})
    assert pd.lengths == {'a': 50, 'b': 6, 'c': 208}
    assert pd.lengths == twin.lengths
    written = torch.zeros(pd.pool_k[0].shape[0], dtype=torch.bool, device=dev())
    for r, c in zip(reqs, counts):
        s0 = pd.slot_rows[pd._slots[r]] + pd.lengths[r] - c
        written[s0:s0 + c] = True
    written[pd.trash_row] = True
    for new, old in zip(pd.pool_k + pd.pool_v, before_k + before_v):
        assert torch.equal(new[~written], old[~written])
    for r in reqs:
        for (a, b), (c, d) in zip(pd.request_kv(r), twin.request_kv(r)):
            assert_bf16_close(a, c.float().cpu().numpy())
            assert_bf16_close(b, d.float().cpu().numpy())
    with pytest.raises(ValueError):
        pd.append_verified(feat, reqs, [0, 9, 0])           # more than the chunk width
    status_clean(pkg)


def test_captured_append_replays_like_eager(pkg):
    draft = build_draft(pkg)
    a = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=300)
    b = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=300)
    g = np.random.Generator(np.random.PCG64(7))
    reqs = tuple(f'q{i}' for i in range(4))
    for pdx in (a, b):
        for r in reqs:
            pdx.add_request(r)
    ctx = {r: features(g, 10 + 20 * i, 1024) for i, r in enumerate(reqs)}
    a.append_committed(ctx)
    b.append_committed(ctx)
    a.capture_append(4, 8)
    for rnd in range(3):
        feat = features(g, 32, 1024)
        counts = [int(c) for c in g.integers(0, 9, 4)]
        a.append_verified_graph(feat, reqs, counts)
        b.append_verified(feat, reqs, counts)
        assert a.lengths == b.lengths
        for x, y in zip(a.pool_k + a.pool_v, b.pool_k + b.pool_v):
            live = torch.ones(x.shape[0], dtype=torch.bool, device=dev())
            live[a.trash_row] = False
            assert torch.equal(x[live], y[live])
    status_clean(pkg)


def test_destination_outside_pool_is_skipped_and_flagged(pkg):
    draft = build_draft(pkg, 256, 2)
    pd = pkg.B200PackedDraft(draft, max_requests=2, context_capacity=64)
    pd.add_request('x')
    before_k, before_v = pools(pd)
    rows = pd.pool_k[0].shape[0]
    context = torch.randn((4, 256), device=dev()).to(torch.bfloat16)
    kv_w, kn_w, rope = pd._append_operands()
    meta = torch.tensor([0, 4, rows - 2, 0, 4], dtype=torch.int32, device=dev())   # rows - 2 + j: j >= 2 outside
    pkg.kernels.draft_append(context, kv_w, kn_w, rope, meta, 1, pd.pool_k, pd.pool_v,
                             pd.trash_row, 1e-6)
    assert pkg.read_device_status(clear=True) & pkg._lib.DEVICE_BAD_ARGUMENT
    for new, old in zip(pd.pool_k + pd.pool_v, before_k + before_v):
        assert torch.equal(new[:rows - 2], old[:rows - 2])
    status_clean(pkg)
