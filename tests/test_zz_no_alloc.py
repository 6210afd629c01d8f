"""The decode-attention entry point that allocates nothing.

Some callers of this library cannot call cudaMalloc at all — a serving host
that reserves the whole GPU into its own pools at start-up, or a
foreign-language binding whose only device allocator is its own tensor pool
and cannot lend scratch for one call.  tb_attention_decode_noalloc_f32 keeps
its split-K partials in a library-owned device array instead.  These tests
call it through the C ABI and check it against tb_attention_f32 (the entry
point with a caller workspace) on two calls in a row, at the attention
tolerance the other tests use.  The file is named so pytest collects it
last, and it needs no state from other tests.
"""
import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # relative to max |out|, as in test_gpu_ops.test_attention


def _case(B, H, Hkv, D, sk, max_seq, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, 1, H, D)).astype(np.float32)
    kc = rng.standard_normal((B, Hkv, max_seq, D)).astype(np.float32)
    vc = rng.standard_normal((B, Hkv, max_seq, D)).astype(np.float32)
    return q, kc, vc


@pytest.mark.parametrize("B,H,Hkv,D,sk,max_seq", [
    (1, 32, 32, 128, 641, 2048),  # the 7B decode shape
    (2, 64, 8, 128, 300, 512),    # 70B grouping: 8 query heads per kv head
    (2, 32, 4, 64, 97, 256),      # 8 query heads per kv head at head_dim 64
    (3, 8, 8, 64, 1, 16),         # a one-key cache
    (16, 64, 8, 128, 2000, 2048),  # one split of partials is 532 KB: fewer splits than the workspace path
])
def test_noalloc_matches_workspace_entry_point(tb, cuda, B, H, Hkv, D, sk, max_seq):
    import torch

    L = tb.lib
    scale = float(ctypes.c_float(1.0 / ctypes.c_float(math.sqrt(D)).value).value)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # two calls in a row share (and reuse) the scratch array
        q, kc, vc = (torch.from_numpy(a).to(cuda) for a in _case(B, H, Hkv, D, sk, max_seq, seed=call + B))
        ws_bytes = L.tb_attention_workspace_size(B, H, 1, D, max_seq)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
        ref = torch.empty_like(q)
        tb.check(L.tb_attention_f32(ref.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, H, Hkv, 1, sk,
                                    D, max_seq, scale, ws.data_ptr(), ws_bytes, stream))
        got = torch.full_like(q, float("nan"))
        tb.check(L.tb_attention_decode_noalloc_f32(got.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), B,
                                                   H, Hkv, sk, D, max_seq, scale, stream))
        torch.cuda.synchronize()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all()
        assert float(np.abs(g - r).max()) <= TOL * float(np.abs(r).max())


def test_noalloc_split_count_is_capped_by_the_scratch(tb):
    """The 16-sequence case above runs with fewer splits than the workspace
    path picks: B * H * (D + 2) * 4 bytes per split fit three times."""
    B, H, D = 16, 64, 128
    per_split = B * H * (D + 2) * 4
    assert 2 * 1024 * 1024 // per_split == 3
    # the workspace entry point sizes for more splits than that
    assert tb.lib.tb_attention_workspace_size(B, H, 1, D, 2048) > 3 * per_split


def test_noalloc_rejects_unsupported_head_grouping(tb, cuda):
    import torch

    # head_dim 32 with 8 query heads per kv head has no decode kernel (as for tb_attention_f32)
    B, H, Hkv, D = 1, 16, 2, 32
    q = torch.zeros((B, 1, H, D), device=cuda)
    kc = torch.zeros((B, Hkv, 8, D), device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = tb.lib.tb_attention_decode_noalloc_f32(q.data_ptr(), q.data_ptr(), kc.data_ptr(), kc.data_ptr(), B, H, Hkv,
                                                4, D, 8, 0.1, st)
    assert rc == tb.TB_ERROR_NOT_SUPPORTED


def test_noalloc_rejects_sizes_beyond_its_scratch(tb, cuda):
    import torch

    # B * H * (D + 2) * 4 bytes for one split exceeds TB_ATTENTION_NOALLOC_SCRATCH_BYTES (2 MiB)
    B, H, D = 64, 64, 128
    q = torch.zeros((B, 1, H, D), device=cuda)
    kc = torch.zeros((B, H, 4, D), device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = tb.lib.tb_attention_decode_noalloc_f32(q.data_ptr(), q.data_ptr(), kc.data_ptr(), kc.data_ptr(), B, H, H,
                                                2, D, 4, 0.1, st)
    assert rc == tb.TB_ERROR_INVALID_ARGUMENT
