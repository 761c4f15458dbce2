"""GPU test of the allocation-free permute entry point, called through its exported C symbol.

Callers such as serving runtimes that reserve all device memory up front, or plain C hosts without a
caching allocator, cannot allocate temporary device buffers per call; `ep_permute_noalloc` keeps its
scratch in a fixed array inside the library. This test calls it twice in a row through ctypes and
checks each result against the regular (allocating) `permute` op: every output must match exactly.
The file sorts last so that a run stopping at its first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from deepep_slingshot_b200._ext import require_ext
    lib = ctypes.CDLL(require_ext().__file__)
    fn = lib.ep_permute_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.ep_permute_noalloc_strerror.restype = ctypes.c_char_p
    lib.ep_permute_noalloc_strerror.argtypes = [ctypes.c_int]
    return fn, lib.ep_permute_noalloc_strerror


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _call(fn, x, xs, probs, idx, E, align, rows):
    N, H = x.shape
    K = idx.shape[1]
    dev = x.device
    out = dict(offsets=torch.full((E + 1,), -7, dtype=torch.int32, device=dev),
               counts=torch.full((E,), -7, dtype=torch.int32, device=dev),
               row_map=torch.full((N, K), -7, dtype=torch.int32, device=dev),
               x_perm=torch.zeros((rows, H), dtype=x.dtype, device=dev),
               scales=torch.zeros((rows, H // 128), dtype=torch.float32, device=dev) if xs is not None else None,
               probs=torch.zeros((rows,), dtype=torch.float32, device=dev) if probs is not None else None)
    rc = fn(_ptr(x), x.element_size(), _ptr(xs), _ptr(probs), _ptr(idx), N, H, K, E, align, _ptr(out['offsets']),
            _ptr(out['counts']), _ptr(out['row_map']), _ptr(out['x_perm']), _ptr(out['scales']), _ptr(out['probs']),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def test_permute_noalloc_matches_permute_twice():
    from deepep_slingshot_b200.ops.permute import permute
    from deepep_slingshot_b200.utils.math import per_token_cast_to_fp8
    fn, strerror = _lib()
    E, K, align = 32, 8, 128
    for call, N in enumerate((1000, 3000)):  # two calls in a row; the second reuses the same scratch
        g = torch.Generator().manual_seed(100 + call)
        x = torch.randn((N, 1024), generator=g).to(torch.bfloat16).cuda()
        idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]).cuda()
        idx[torch.rand((N, K), generator=g).cuda() < 0.1] = -1
        w = torch.rand((N, K), generator=g).cuda()
        xq, xs = per_token_cast_to_fp8(x)
        ref = permute(xq, idx, E, alignment=align, probs=w, x_scales=xs)
        rows = ref.x.shape[0]
        rc, out = _call(fn, xq, xs, w, idx, E, align, rows)
        torch.cuda.synchronize()
        assert rc == 0, strerror(rc)
        assert torch.equal(out['offsets'], ref.expert_offsets)
        assert torch.equal(out['counts'], ref.expert_counts)
        assert torch.equal(out['row_map'], ref.row_map)
        used = int(ref.expert_offsets[-1])
        valid_rows = ref.row_map[ref.row_map >= 0].long()
        assert torch.equal(out['x_perm'][valid_rows].view(torch.uint8), ref.x[valid_rows].view(torch.uint8))
        assert torch.equal(out['scales'][valid_rows], ref.scales[valid_rows])
        assert torch.equal(out['probs'][:used], ref.probs[:used])


def test_permute_noalloc_rejects_oversize():
    fn, strerror = _lib()
    N, E = 32 * 4096, 64  # 4096 chunks * 64 experts > the fixed scratch
    x = torch.zeros((N, 128), dtype=torch.bfloat16, device='cuda')
    idx = torch.zeros((N, 1), dtype=torch.int64, device='cuda')
    rc, _ = _call(fn, x, None, None, idx, E, 1, 16)
    assert rc == 2 and b'too large' in strerror(rc)
