"""The allocation-free attention entry point (qw_attention_noalloc) against qw_attention.

qw_attention_noalloc exists for callers that cannot allocate device memory per call (a
host runtime that owns all device memory through its own pool, or a thread on which a
cudaMalloc would synchronise the device): its split-K scratch is a fixed array inside
the library instead of a caller workspace.  Both entry points are called through the C
ABI on the same inputs; two calls in a row with different shapes and dtypes check that
the second call is not disturbed by what the first left in the shared array.  The file
is named so that pytest collects it last.
"""
import numpy as np
import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu

# (dtype, batch, heads, kv_heads, seq, query_start, dim): the first is the target's
# attention block (16 query / 2 KV heads of 256, a 16-token block over 1024 keys)
CASES = [(torch.bfloat16, 1, 16, 2, 16, 1024, 256), (torch.float16, 3, 8, 8, 5, 295, 128)]


def _inputs(rng, dtype, b, h, hkv, s, qs, d):
    def t(*shape):
        return torch.from_numpy(rng.normal(0, 1, shape).astype(np.float32)).to("cuda", dtype)
    return t(b, h, s, d), t(b, hkv, qs + s, d), t(b, hkv, qs + s, d)


def _call_both(so, lib, q, k, v, dtype, b, h, hkv, s, qs, d):
    scale = d ** -0.5
    code = lib.dtype_code(dtype)
    total = qs + s
    want = torch.empty_like(q)
    ws = torch.empty(so.qw_attn_workspace_bytes(b, h, hkv, s, d, total), dtype=torch.uint8, device="cuda")
    lib.check(so.qw_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), want.data_ptr(), code, b, h, hkv, s,
                              total, d, qs, scale, ws.data_ptr(), None), "qw_attention")
    got = torch.full_like(q, float("nan"))
    lib.check(so.qw_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(), code, b, h, hkv,
                                      s, total, d, qs, scale, None), "qw_attention_noalloc")
    torch.cuda.synchronize()
    return got.float().cpu().numpy(), want.float().cpu().numpy()


def test_noalloc_attention_matches_workspace_entry_point_twice(cuda_lib):
    from qwen35_dflash_b200 import lib
    so = lib.load()
    rng = np.random.default_rng(23)
    for case in CASES:
        dtype, b, h, hkv, s, qs, d = case
        need = so.qw_attn_workspace_bytes(b, h, hkv, s, d, qs + s)
        assert 0 < need <= lib.QW_ATTN_NOALLOC_SCRATCH_BYTES, (case, need)
        q, k, v = _inputs(rng, dtype, b, h, hkv, s, qs, d)
        got, want = _call_both(so, lib, q, k, v, dtype, b, h, hkv, s, qs, d)
        assert np.isfinite(got).all(), case
        assert_close(got, want, what=f"attention_noalloc {case}")


def test_noalloc_attention_rejects_shapes_beyond_its_scratch(cuda_lib):
    from qwen35_dflash_b200 import lib
    so = lib.load()
    b, h, hkv, s, qs, d = 64, 16, 2, 16, 4096, 256
    assert so.qw_attn_workspace_bytes(b, h, hkv, s, d, qs + s) > lib.QW_ATTN_NOALLOC_SCRATCH_BYTES
    q = torch.zeros(b, h, s, d, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(b, hkv, qs + s, d, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(q)
    with pytest.raises(ValueError, match="scratch"):
        lib.check(so.qw_attention_noalloc(q.data_ptr(), k.data_ptr(), k.data_ptr(), out.data_ptr(),
                                          lib.QW_BF16, b, h, hkv, s, qs + s, d, qs, d ** -0.5, None),
                  "qw_attention_noalloc")
    assert not out.any()
