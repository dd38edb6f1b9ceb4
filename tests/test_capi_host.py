"""C-ABI library and host-side contract checks that need no GPU.

* the shared library loads and exports every function include/dspark_b200.h declares;
* argument checks that need no device run before any launch (status, not a crash);
* the drop-in kernel classes refuse the reference's contract violations before the
  native entry is called, pass the reference's argument meaning to it, cache layout
  validation per layout object and propagate native failures without fallback
  (the shape of the reference's tests/test_rocm_varlen.py, with the entry mocked).
"""
import ctypes
import os
import re
from unittest.mock import Mock, PropertyMock, patch

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, 'include', 'dspark_b200.h')).read()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(dspark_\w+)\s*\(', text)))


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    raw = ctypes.CDLL(pkg.LIB_PATH)
    names = header_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(raw, name), name
    assert lib.dspark_abi_version() == 18
    assert lib.dspark_status_string(1) == b'invalid argument'
    assert pkg.launch_count() >= 0


def test_null_arguments_are_refused_before_any_device_work(pkg):
    lib = pkg.load_library()
    st = lib.dspark_varlen_attn(None, None, None, None, None, 1, 1, 1, 1, 1, 128 ** -0.5, 0, None, None, 0, None)
    assert st == 1
    st = lib.dspark_commit_kv(None, None, None, None, None, None, None, None, None, 1, 1, 1, 1, 0, None)
    assert st == 1
    assert lib.dspark_rope_table(None, 8, None, None, 1, 1, None, None) == 1
    fake = ctypes.c_void_p(256)
    assert lib.dspark_rope_table(fake, 0, fake, fake, 1, 1, fake, None) == 1          # empty cache
    assert lib.dspark_rope_table(ctypes.c_void_p(264), 8, fake, fake, 1, 1, fake, None) == 1   # unaligned cache
    size = ctypes.c_size_t(0)
    assert lib.dspark_attention_workspace_size(0, None) == 1
    # training layout, acceptance and Markov entries refuse before touching the device
    assert lib.dspark_train_attn(None, None, None, 1, 1, None, 1, 128 ** -0.5, None, None) == 1
    assert lib.dspark_row_argmax(None, 16, 1, 16, 0, None, None) == 1
    assert lib.dspark_row_argmax(ctypes.c_void_p(16), 8, 1, 16, 0, ctypes.c_void_p(16), None) == 1   # ld < vocab
    assert lib.dspark_greedy_accept(None, None, None, 1, 1, None, 0, None, None, None, None, None) == 1
    # bf16 RMSNorm: null pointers, hidden not a multiple of 8, short or unaligned strides, misaligned rows
    fake16 = ctypes.c_void_p(256)
    assert lib.dspark_rms_norm(None, 1024, fake16, 1e-6, 4, 1024, fake16, 1024, None) == 1
    for ld_x, hidden, ld_out, ptr in ((1020, 1020, 1020, 256), (512, 1024, 1024, 256), (1028, 1024, 1024, 256),
                                      (1024, 1024, 1024, 258)):
        p = ctypes.c_void_p(ptr)
        assert lib.dspark_rms_norm(p, ld_x, fake16, 1e-6, 4, hidden, fake16, ld_out, None) == 1
    assert lib.dspark_rms_norm(fake16, 1024, fake16, -1.0, 4, 1024, fake16, 1024, None) == 1   # negative eps
    assert lib.dspark_rms_norm(fake16, 1024, fake16, 1e-6, 0, 1024, fake16, 1024, None) == 0    # no rows: no launch
    assert lib.dspark_add_rms_norm(fake16, 1024, None, 1024, fake16, 1e-6, 4, 1024, fake16, 1024, fake16, 1024,
                                   None) == 1                                                  # null delta
    assert lib.dspark_add_rms_norm(fake16, 1024, fake16, 1020, fake16, 1e-6, 4, 1024, fake16, 1024, fake16, 1024,
                                   None) == 1                                                  # short stride
    assert lib.dspark_add_rms_norm(None, 1024, None, 1024, None, 1e-6, 0, 1024, None, 1024, None, 1024, None) == 0
    # outputs that share bytes with an input, or with each other, are refused: the second
    # pass re-reads x and delta after the stores (4 rows x 1024 bf16 = 8 KiB spans)
    x, d, o, s = (ctypes.c_void_p(a) for a in (0x100000, 0x200000, 0x300000, 0x400000))
    for args in ((x, d, o, x), (x, d, d, s), (x, d, o, ctypes.c_void_p(0x100000 + 6 * 1024)),
                 (x, d, ctypes.c_void_p(0x200000 + 2048 * 3), s), (x, d, o, ctypes.c_void_p(0x300000 + 2048))):
        xa, da, oa, sa = args
        assert lib.dspark_add_rms_norm(xa, 1024, da, 1024, fake16, 1e-6, 4, 1024, oa, 1024, sa, 1024, None) == 1
    # draft q/k norm + RoPE: strides shorter than the heads, unaligned pointers, null pointers
    f = ctypes.c_void_p(256)
    assert lib.dspark_qk_norm_rope(f, 2000, f, 1024, f, f, 1e-6, 1e-6, f, f, 128, 4, 16, 8, f, f, None) == 1
    assert lib.dspark_qk_norm_rope(f, 2048, f, 1024, f, f, 1e-6, 1e-6, f, f, 64, 4, 16, 8, f, f, None) == 1
    assert lib.dspark_qk_norm_rope(ctypes.c_void_p(258), 2048, f, 1024, f, f, 1e-6, 1e-6, f, f, 128, 4, 16, 8, f,
                                   f, None) == 1
    assert lib.dspark_qk_norm_rope(None, 2048, f, 1024, f, f, 1e-6, 1e-6, f, f, 128, 4, 16, 8, f, f, None) == 1
    # merged gate/up activation: stride shorter than both halves, inter not a multiple of 8, null, misaligned
    assert lib.dspark_silu_mul(f, 3000, 4, 1536, f, 1536, None) == 1
    assert lib.dspark_silu_mul(f, 3072, 4, 1532, f, 1532, None) == 1
    assert lib.dspark_silu_mul(None, 3072, 4, 1536, f, 1536, None) == 1
    assert lib.dspark_silu_mul(f, 3072, 4, 1536, ctypes.c_void_p(264), 1536, None) == 1
    assert lib.dspark_silu_mul(None, 3072, 0, 1536, None, 1536, None) == 0
    assert lib.dspark_qk_norm_rope(None, 2048, None, 1024, None, None, 1e-6, 1e-6, None, None, 128, 0, 16, 8, None,
                                   None, None) == 0
    assert lib.dspark_markov_step(None, None, 1024, 256, None, 7, 0, None, 1, None, 1024, None, 0.0, None, None, 7, 1,
                                  None, None) == 1
    fake = ctypes.c_void_p(256)
    for vocab, rank, r in ((1001, 256, 4), (1024, 96, 4), (1024, 320, 4), (1024, 256, 129)):   # refused shapes
        assert lib.dspark_markov_step(fake, fake, vocab, rank, fake, 7, 0, fake, 1, fake, 1024, fake, 0.0, fake,
                                      fake, 7, r, fake, None) == 1
    # the block entry: block sizes 1..64, the same operand rules, anchors required
    for vocab, rank, r, bs in ((1001, 256, 4, 7), (1024, 96, 4, 7), (1024, 256, 129, 7), (1024, 256, 4, 0),
                               (1024, 256, 4, 65)):
        assert lib.dspark_markov_block(fake, fake, vocab, rank, fake, bs, fake, fake, 1024, fake, 0.0, fake, fake, r,
                                       fake, None) == 1
    assert lib.dspark_markov_block(fake, fake, 1024, 256, fake, 7, None, fake, 1024, fake, 0.0, fake, fake, 4, fake,
                                   None) == 1
    assert lib.dspark_markov_scratch_bytes() >= 3 * 128 * 8 + 8
    # stochastic acceptance: target rows must be draft rows + requests, temperature > 0
    for rows, temp in ((4, 1.0), (3, 0.0), (3, float('nan'))):
        assert lib.dspark_stochastic_accept(fake, 1000, 1, 1000, temp, rows, fake, 1, fake, fake, 2, fake, 2, None, 0,
                                            fake, fake, fake, fake, 1 << 20, None) == 1
    assert lib.dspark_stochastic_accept(None, 1000, 1, 1000, 1.0, 3, fake, 1, fake, fake, 2, fake, 2, None, 0, fake,
                                        fake, fake, fake, 1 << 20, None) == 1
    assert lib.dspark_stochastic_scratch_bytes(4) >= 4 * 24
    ptrs = (ctypes.c_void_p * 1)(256)
    assert lib.dspark_draft_append(None, 8, 1024, fake, 1, fake, fake, 1e-6, fake, fake, fake, fake, 1, ptrs, ptrs,
                                   16, 15, None) == 1
    for rows, hidden, layers, trash in ((8, 1000, 1, 15), (8, 1024, 9, 15), (0, 1024, 1, 15), (8, 1024, 1, 16)):
        assert lib.dspark_draft_append(fake, rows, hidden, fake, layers, fake, fake, 1e-6, fake, fake, fake, fake, 1,
                                       ptrs, ptrs, 16, trash, None) == 1
    nul = (ctypes.c_void_p * 1)(None)
    assert lib.dspark_draft_append(fake, 8, 1024, fake, 1, fake, fake, 1e-6, fake, fake, fake, fake, 1, nul, ptrs,
                                   16, 15, None) == 1
    # the k_norm weights are read as 16-byte vectors
    assert lib.dspark_draft_append(fake, 8, 1024, fake, 1, ctypes.c_void_p(264), fake, 1e-6, fake, fake, fake, fake, 1, ptrs,
                                   ptrs, 16, 15, None) == 1


def _fixture(pkg):
    q = torch.zeros(9, 16, 128, dtype=torch.bfloat16)
    k = torch.zeros(46, 8, 128, dtype=torch.bfloat16)
    layout = pkg.PackedLayout((1, 2), (1, 8), (17, 29), torch.tensor([0, 1, 9], dtype=torch.int32),
                              torch.tensor([0, 17, 46], dtype=torch.int32), torch.arange(46), 46)
    return q, k, k.clone(), layout


def _kernel(pkg, cls):
    with patch.object(pkg.kernels, 'runtime_identity', return_value={'device': 'fake'}) as ident:
        kern = cls(torch.device('cpu'))
    ident.assert_called_once()
    kern._operator = Mock()
    return kern


@pytest.mark.parametrize('name,causal_entry', [('B200VarlenKernel', 'dspark_varlen_attn'),
                                               ('B200DraftKernel', 'dspark_draft_attn')])
def test_entry_arguments_and_layout_cache(pkg, name, causal_entry):
    cls = getattr(pkg, name)
    assert cls.entry == causal_entry and cls.native_varlen_calls_per_layer == 1
    q, k, v, layout = _fixture(pkg)
    kern = _kernel(pkg, cls)
    with patch.object(torch.Tensor, 'is_cuda', new_callable=PropertyMock, return_value=True), \
            patch.object(pkg.kernels._lib, 'workspace', return_value=torch.zeros(16, dtype=torch.uint8)), \
            patch.object(pkg.kernels, '_stream', return_value=0):
        kern(q, k, v, layout, scale=128 ** -0.5)
        kern(q, k, v, layout, scale=128 ** -0.5)
        assert kern._operator.call_count == 2
        args = kern._operator.call_args[0]
        # (q, k, v, cu_q, cu_k, R, total_q, key_rows, max_q, max_k, scale, dtype, out, ws, ws_bytes, stream)
        assert args[5:12] == (2, 9, 46, 8, 29, 128 ** -0.5, 0)
        assert kern._validated_layout is layout
        layout.cu_query[1] = 2
        with pytest.raises(ValueError, match='Cumulative lengths'):
            kern(q, k, v, layout, scale=128 ** -0.5)
    assert kern._operator.call_count == 2


def test_contract_violations_refused_before_entry(pkg):
    for mutation in ['dtype', 'heads', 'scale', 'cu_dtype', 'noncontiguous', 'tokens', 'requires_grad', 'q_gt_k']:
        q, k, v, layout = _fixture(pkg)
        kern = _kernel(pkg, pkg.B200VarlenKernel)
        scale = 128 ** -0.5
        if mutation == 'dtype':
            q = q.half()
        if mutation == 'requires_grad':
            q = q.float().requires_grad_(True)
        if mutation == 'heads':
            q = q[:, :8].contiguous()
        if mutation == 'scale':
            scale = 1.0
        if mutation == 'cu_dtype':
            object.__setattr__(layout, 'cu_query', layout.cu_query.long())
        if mutation == 'noncontiguous':
            q = torch.zeros(9, 16, 256, dtype=torch.bfloat16)[:, :, ::2]
        if mutation == 'tokens':
            q = q[:1]
        if mutation == 'q_gt_k':
            layout = pkg.PackedLayout((1, 2), (1, 8), (17, 7), torch.tensor([0, 1, 9], dtype=torch.int32),
                                      torch.tensor([0, 17, 24], dtype=torch.int32), torch.arange(24), 24)
            k, v = k[:24].contiguous(), v[:24].contiguous()
        with patch.object(torch.Tensor, 'is_cuda', new_callable=PropertyMock, return_value=True):
            with pytest.raises(ValueError):
                kern(q, k, v, layout, scale=scale)
        kern._operator.assert_not_called()


def test_native_failure_propagates_without_fallback(pkg):
    kern = _kernel(pkg, pkg.B200VarlenKernel)
    kern._operator.side_effect = RuntimeError('native fixture failure')
    with patch.object(torch.Tensor, 'is_cuda', new_callable=PropertyMock, return_value=True), \
            patch.object(pkg.kernels._lib, 'workspace', return_value=torch.zeros(16, dtype=torch.uint8)), \
            patch.object(pkg.kernels, '_stream', return_value=0):
        with pytest.raises(RuntimeError, match='native fixture failure'):
            kern(*_fixture(pkg), scale=128 ** -0.5)


def test_constructor_refuses_cpu_device(pkg):
    with pytest.raises(RuntimeError, match='no CPU fallback'):
        pkg.B200DraftKernel(torch.device('cpu'))


def test_capacity_kernel_requires_capacity_rows(pkg):
    kern = _kernel(pkg, pkg.B200CapacityKernel)
    q = torch.zeros(9, 16, 128, dtype=torch.bfloat16)
    k = torch.zeros(50, 8, 128, dtype=torch.bfloat16)
    lay = pkg.PersistentAttentionLayout((1, 8), (17, 29), torch.tensor([0, 1, 9], dtype=torch.int32),
                                        torch.tensor([0, 17, 46], dtype=torch.int32), 50, 29, 8)
    bad = pkg.PersistentAttentionLayout((1, 8), (17, 29), lay.cu_query, lay.cu_key, 49, 29, 8)
    with patch.object(torch.Tensor, 'is_cuda', new_callable=PropertyMock, return_value=True), \
            patch.object(pkg.kernels._lib, 'workspace', return_value=torch.zeros(16, dtype=torch.uint8)), \
            patch.object(pkg.kernels, '_stream', return_value=0):
        with pytest.raises(ValueError):
            kern(q, k, k.clone(), bad, scale=128 ** -0.5)
        kern(q, k, k.clone(), lay, scale=128 ** -0.5)
        assert kern._operator.call_args[0][7] == 50      # key_rows = capacity; the tail is never read


def test_packed_layout_mirror_matches_reference_fixture(pkg, golden):
    for idx in (0, 1):
        g = golden(f'layout{idx}')
        L = lambda x: torch.tensor(x.tolist(), dtype=torch.long)  # noqa: E731
        lay = pkg.PackedLayout.from_metadata(L(g['qr']), L(g['qp']), L(g['kr']), L(g['kp']))
        assert lay.request_markers == tuple(g['markers'].tolist())
        assert lay.query_lengths == tuple(g['query_lengths'].tolist())
        assert lay.key_lengths == tuple(g['key_lengths'].tolist())
        assert lay.cu_query.tolist() == g['cu_query'].tolist()
        assert lay.cu_key.tolist() == g['cu_key'].tolist()
        assert lay.gather_indices.tolist() == g['gather'].tolist()
        assert lay.pair_domain == int(g['pair_domain'])
    for qreq, qpos, kreq, kpos in [([1, 2, 1], [0, 0, 1], [1, 1, 2], [0, 1, 0]), ([1], [0], [1, 1], [0, 1]),
                                   ([1], [1], [1, 1], [0, 2]), ([], [], [], [])]:
        with pytest.raises(ValueError):
            pkg.PackedLayout.from_metadata(*(torch.tensor(x, dtype=torch.long) for x in [qreq, qpos, kreq, kpos]))


def test_gather_kv_packs_the_layout_rows(pkg, golden):
    """``gather_kv`` returns, request after request, the cache rows the layout names as
    [sum K, Hkv, D] (checked element-wise against the cache), and refuses mismatched pairs."""
    g = golden('layout1')
    L = lambda x: torch.tensor(x.tolist(), dtype=torch.long)  # noqa: E731
    lay = pkg.PackedLayout.from_metadata(L(g['qr']), L(g['qp']), L(g['kr']), L(g['kp']))
    n = lay.physical_key_tokens
    key = torch.randn((1, 8, n, 128))
    value = torch.randn((1, 8, n, 128))
    k, v = lay.gather_kv(key, value)
    assert k.shape == v.shape == (lay.gathered_key_tokens, 8, 128) and k.is_contiguous()
    for packed_row, cache_row in enumerate(g['gather'].tolist()):
        assert torch.equal(k[packed_row], key[0, :, cache_row])
        assert torch.equal(v[packed_row], value[0, :, cache_row])
    for bad_k, bad_v in ((key[:, :, :-1], value[:, :, :-1]), (key, value.double()), (key[0], value[0]),
                         (key, value[:, :4])):
        with pytest.raises(ValueError):
            lay.gather_kv(bad_k, bad_v)


def test_noalloc_entry_size_and_refusals(pkg):
    """The allocation-free verify entry: its static scratch is the workspace of 148 CTAs
    (two fp32 partial slots of 8 heads x 16 rows x 128 d plus their (m, l) pairs, eight
    48-byte merge records and a tile range per CTA), and bad arguments are refused before
    any device work."""
    lib = pkg.load_library()
    lib.dspark_varlen_attn_noalloc_scratch_bytes.restype = ctypes.c_size_t
    per_cta = 2 * (8 * 16 * 128 + 8 * 16 * 2) * 4 + 8 * 48 + 2 * 8
    assert lib.dspark_varlen_attn_noalloc_scratch_bytes() == 148 * per_cta
    fn = lib.dspark_varlen_attn_noalloc
    vp = ctypes.c_void_p
    fn.restype = ctypes.c_int
    fn.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, vp, vp]
    f = vp(256)
    good = [f, f, f, f, f, 1, 7, 64, 7, 64, 128 ** -0.5, f, None]
    for i, bad in ((1, None), (2, None), (4, None), (7, 0), (5, 0), (6, 0), (10, 0.0), (0, vp(258))):
        args = list(good)
        args[i] = bad
        assert fn(*args) == 1, (i, bad)
