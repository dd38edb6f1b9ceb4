"""The allocation-free verify attention entry point, checked against the workspace entry point.

dspark_varlen_attn_noalloc serves callers that cannot allocate device memory for
a workspace: a host that reaches this library through a C FFI and has no access
to the allocator that owns the GPU, or a server whose KV-cache pool already holds
nearly all HBM. Its scratch is a static device array inside the library that
keeps the previous call's contents, so the test makes two calls in a row on
different inputs and compares each, through the C ABI, with dspark_varlen_attn
(caller-provided workspace) on the same inputs: on a 148-SM B200 both launch the same
kernel on the same grid, so the outputs must be identical bit for bit; each output
also meets the bf16 gate against the oracle's bottom-right attention. The documented
scratch size and the argument refusals are checked without a GPU in test_capi_host.py.
"""
import ctypes

import pytest
import torch

import inputs as I
from gpu_util import assert_bf16_close, dev, status_clean, to_dev
from oracle import bottom_right_varlen

pytestmark = pytest.mark.gpu


def _noalloc_entry(lib):
    fn = lib.dspark_varlen_attn_noalloc
    vp = ctypes.c_void_p
    fn.restype = ctypes.c_int
    fn.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, vp, vp]
    return fn


def test_noalloc_matches_workspace_entry_on_two_calls(pkg):
    torch.cuda.set_device(0)
    lib = pkg.load_library()
    fn = _noalloc_entry(lib)
    lib.dspark_varlen_attn_noalloc_scratch_bytes.restype = ctypes.c_size_t
    assert lib.dspark_varlen_attn_noalloc_scratch_bytes() > 0
    pkg.read_device_status(clear=True)
    kernel = pkg.B200VarlenKernel(dev())
    # Call 1 splits one long request over every CTA (partials + merge use the
    # scratch); call 2 has different lengths, so stale call-1 scratch would show.
    cases = [((7, 7, 3, 8), (30000, 57, 10, 1031), 41), ((8, 1, 7), (2000, 5, 12000), 42)]
    for qlens, klens, seed in cases:
        q, k, v = I.varlen_case(seed, qlens, klens, True)
        qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
        layout = pkg.PackedLayout.from_lengths(qlens, klens, dev())
        expected = kernel(qd, kd, vd, layout, scale=I.SCALE)
        out = torch.empty_like(qd)
        status = fn(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), layout.cu_query.data_ptr(),
                    layout.cu_key.data_ptr(), len(qlens), qd.shape[0], kd.shape[0], max(qlens), max(klens),
                    I.SCALE, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert status == 0, lib.dspark_status_string(status)
        torch.cuda.synchronize()
        if torch.cuda.get_device_properties(0).multi_processor_count == 148:
            assert torch.equal(out.view(torch.int16), expected.view(torch.int16))
        assert_bf16_close(out, bottom_right_varlen(q, k, v, qlens, klens, I.SCALE))
        assert_bf16_close(expected, bottom_right_varlen(q, k, v, qlens, klens, I.SCALE))
    status_clean(pkg)
