"""GPU parity of the verify layer (QK-norm + RoPE + KV append + attention) and commit/rollback,
through both the fused kernel and the prep-kernel path.

Checked against the oracle: ``qk_norm_rope_bf16`` for the appended K (bit-exact:
the oracle equals transformers' CPU evaluation bit for bit, and the kernels use its
summation order and its cos/sin), the two-source bottom-right attention for the
output, and ``OracleKVStore.commit`` for the resident state after commit
(bit-exact: commit is a byte copy).
"""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import assert_bf16_close, dev, status_clean
from oracle import OracleKVStore, bf16_bits_to_f32, f32_to_bf16_bits, qk_norm_rope_bf16, two_segment_attention

pytestmark = pytest.mark.gpu


def bits_to_dev(bits):
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16).to(dev())


def dev_to_bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().astype(np.uint16)


def make_store(pkg, layers, caps, max_q, g):
    store = pkg.B200PersistentTargetKV(layers=layers, slots=len(caps), context_capacity=max(caps),
                                       max_query_tokens=max_q, device=dev(), slot_capacities=caps)
    oracle = OracleKVStore(layers, len(caps), max(caps), max_q, 8, 128, np.float32)
    return store, oracle


@pytest.mark.parametrize('path', ['fused', 'prep'])
@pytest.mark.parametrize('weights', ['ones', 'random'])
def test_fused_verify_commit_rollback(pkg, weights, path):
    g = I.rng(7 if weights == 'ones' else 8)
    layers = 3
    contexts = [0, 1, 300, 2047, 64]
    qlens = [7, 7, 3, 8, 7]
    caps = [c + 16 for c in contexts]
    store, _ = make_store(pkg, layers, caps, sum(qlens), g)
    handles = [store.add_request(f'r{i}') for i in range(len(contexts))]
    res_k, res_v = {}, {}
    for h, c in zip(handles, contexts):
        kb = f32_to_bf16_bits(I.normal(g, (layers, c, 8, 128)))
        vb = f32_to_bf16_bits(I.normal(g, (layers, c, 8, 128)))
        res_k[h.index], res_v[h.index] = kb, vb
        if c:
            store.load_prefix(h, bits_to_dev(kb), bits_to_dev(vb))
    nq = sum(qlens)
    tx = store.begin(handles, query_lengths=qlens)
    inv = pkg.rope_inv_freq(I.ROPE_THETA, device=dev())
    positions = np.concatenate([np.arange(c, c + q) for c, q in zip(contexts, qlens)])
    staged_k, staged_v = [], []
    for layer in range(layers):
        qr = f32_to_bf16_bits(I.normal(g, (nq, 16, 128)) * 2)
        kr = f32_to_bf16_bits(I.normal(g, (nq, 8, 128)) * 2)
        vr = f32_to_bf16_bits(I.normal(g, (nq, 8, 128)))
        if weights == 'ones':
            qw = kw = f32_to_bf16_bits(np.ones(128, np.float32))
        else:
            qw = f32_to_bf16_bits(1 + 0.1 * I.normal(g, (128,)))
            kw = f32_to_bf16_bits(1 + 0.1 * I.normal(g, (128,)))
        out = store.verify_layer(tx, layer, bits_to_dev(qr), bits_to_dev(kr), bits_to_dev(vr), bits_to_dev(qw),
                                 bits_to_dev(kw), inv_freq=inv, eps=I.RMS_EPS, path=path)
        torch.cuda.synchronize()
        q_o, k_o = qk_norm_rope_bf16(qr, kr, qw, kw, positions, I.ROPE_THETA, I.RMS_EPS)
        # KV append: scratch rows hold roped k and raw v of this layer.
        sk = dev_to_bits(store.scratch_keys[layer * store.max_query_tokens:][:nq])
        sv = dev_to_bits(store.scratch_values[layer * store.max_query_tokens:][:nq])
        assert np.array_equal(sv, vr)
        assert np.array_equal(sk, k_o)          # the reference's CPU k_norm + RoPE, bit for bit
        staged_k.append(sk)
        staged_v.append(sv)
        # attention over resident prefix + own new rows
        segs, qo = [], 0
        for h, c, q in zip(handles, contexts, qlens):
            rk = bf16_bits_to_f32(res_k[h.index][layer]) if c else np.zeros((0, 8, 128), np.float32)
            rv = bf16_bits_to_f32(res_v[h.index][layer]) if c else np.zeros((0, 8, 128), np.float32)
            segs.append(((rk, rv, 0, c), (bf16_bits_to_f32(sk), bf16_bits_to_f32(sv), qo, q)))
            qo += q
        assert_bf16_close(out, two_segment_attention(bf16_bits_to_f32(q_o), qlens, segs, I.SCALE, True))
    # commit accepted prefixes (anchor included); the rest is rolled back
    accept = [1, 7, 0, 5, 3]
    result = store.commit(tx, {h: n for h, n in zip(handles, accept)})
    torch.cuda.synchronize()
    assert result['committed_tokens'] == sum(accept)
    qo = 0
    for h, c, q, n in zip(handles, contexts, qlens, accept):
        assert store.length(h) == c + n
        k_now, v_now = store.request_kv(h)
        want_k = np.concatenate([res_k[h.index], np.stack([s[qo:qo + n] for s in staged_k])], axis=1)
        want_v = np.concatenate([res_v[h.index], np.stack([s[qo:qo + n] for s in staged_v])], axis=1)
        assert np.array_equal(dev_to_bits(k_now), want_k)
        assert np.array_equal(dev_to_bits(v_now), want_v)
        qo += q
    # second round sees the grown contexts; abort leaves resident bytes untouched
    before = store.keys.clone()
    tx2 = store.begin(handles, query_lengths=[1] * len(handles))
    store.abort(tx2)
    assert torch.equal(before, store.keys)
    status_clean(pkg)


def test_commit_matches_oracle_store_uniform_layout(pkg):
    """Uniform capacities: resident memory equals the reference's [L, slots, C, H, D] after commit."""
    g = I.rng(12)
    layers, slots, cap, maxq = 2, 3, 24, 8
    store = pkg.B200PersistentTargetKV(layers=layers, slots=slots, context_capacity=cap, max_query_tokens=maxq,
                                       device=dev())
    oracle = OracleKVStore(layers, slots, cap, maxq, 8, 128, np.uint16)
    hs = [store.add_request(n) for n in ('A', 'B', 'idle')]
    for s, n in zip(range(3), (3, 5, 9)):
        kb = f32_to_bf16_bits(I.normal(g, (layers, n, 8, 128)))
        vb = f32_to_bf16_bits(I.normal(g, (layers, n, 8, 128)))
        store.load_prefix(hs[s], bits_to_dev(kb), bits_to_dev(vb))
        oracle.load_prefix(s, kb, vb)
    tx = store.begin(hs[:2], query_lengths=(2, 3))
    for layer in range(layers):
        kb = f32_to_bf16_bits(I.normal(g, (5, 8, 128)))
        vb = f32_to_bf16_bits(I.normal(g, (5, 8, 128)))
        store.stage_layer(tx, layer, bits_to_dev(kb), bits_to_dev(vb))
        oracle.stage_layer(layer, kb, vb)
    store.commit(tx, {hs[0]: 1, hs[1]: 2})
    oracle.commit([0, 1], [3, 5], [2, 3], [1, 2])
    torch.cuda.synchronize()
    assert np.array_equal(dev_to_bits(store.keys), oracle.keys)
    assert np.array_equal(dev_to_bits(store.values), oracle.values)
    assert [store.length(h) for h in hs] == oracle.lengths
    status_clean(pkg)


def test_store_refusals(pkg):
    store = pkg.B200PersistentTargetKV(layers=1, slots=2, context_capacity=8, max_query_tokens=4, device=dev())
    a = store.add_request('A')
    with pytest.raises(ValueError):
        store.begin([a], query_lengths=(9,))
    tx = store.begin([a], query_lengths=(2,))
    with pytest.raises(RuntimeError):
        store.add_request('B')
    with pytest.raises(ValueError):
        store.commit(tx, {a: 1})            # layer not staged
    z = torch.zeros((2, 8, 128), dtype=torch.bfloat16, device=dev())
    store.stage_layer(tx, 0, z, z)
    with pytest.raises(ValueError):
        store.commit(tx, {a: 3})
    with pytest.raises(ValueError):
        store.commit(tx, {a: True})
    store.commit(tx, {a: 0})
    assert store.length(a) == 0
    with pytest.raises(ValueError):
        store.abort(tx)


def test_strided_projection_rows_equal_packed_rows(pkg):
    """q/k/v as column blocks of one merged [n, 4096] projection (row stride 4096, the
    target's single q|k|v GEMM) give the packed inputs' output and scratch K/V bit for
    bit on the prep path; 'auto' takes the prep path for them and 'fused' refuses them."""
    g = I.rng(21)
    contexts, qlens = [5, 600, 0], [8, 8, 8]
    caps = [c + 16 for c in contexts]
    nq = sum(qlens)
    inv = pkg.rope_inv_freq(I.ROPE_THETA, device=dev())
    qkv = bits_to_dev(f32_to_bf16_bits(I.normal(g, (nq, 32 * 128)) * 2))
    qw = bits_to_dev(f32_to_bf16_bits(1 + 0.1 * I.normal(g, (128,))))
    kw = bits_to_dev(f32_to_bf16_bits(1 + 0.1 * I.normal(g, (128,))))
    q = qkv[:, :2048].view(nq, 16, 128)
    k = qkv[:, 2048:3072].view(nq, 8, 128)
    v = qkv[:, 3072:].view(nq, 8, 128)
    results = []
    for strided in (False, True):
        store, _ = make_store(pkg, 1, caps, nq, g)
        handles = [store.add_request(f'r{i}') for i in range(3)]
        for h, c in zip(handles, contexts):
            if c:
                kv = bits_to_dev(f32_to_bf16_bits(I.normal(I.rng(30 + c), (2, 1, c, 8, 128))))
                store.load_prefix(h, kv[0], kv[1])
        tx = store.begin(handles, query_lengths=qlens)
        args = (q, k, v) if strided else (q.contiguous(), k.contiguous(), v.contiguous())
        if strided:
            with pytest.raises(ValueError):
                store.verify_layer(tx, 0, *args, qw, kw, inv_freq=inv, eps=I.RMS_EPS, path='fused')
        out = store.verify_layer(tx, 0, *args, qw, kw, inv_freq=inv, eps=I.RMS_EPS,
                                 path='auto' if strided else 'prep')
        torch.cuda.synchronize()
        results.append((out.clone(), store.scratch_keys[:nq].clone(), store.scratch_values[:nq].clone()))
        store.abort(tx)
    for a, b in zip(*results):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    status_clean(pkg)
