"""The allocation-free decode attention entry point.

Callers such as engines with a fixed, pre-reserved memory pool, or hosts that
forbid device allocation on their inference thread, cannot hand the library a
workspace.  vmlx_cuda_sdpa_decode_noalloc keeps its partials in a fixed array
inside the library instead.  This test calls it through the C ABI twice in a
row (different inputs, so a stale first result would show) and checks each
result against the workspace-taking vmlx_cuda_sdpa_decode on the same inputs,
within the matmul tolerance of the other tests (max rel 1e-2).  It also checks
that sizes beyond the built-in scratch are rejected.  The file is named to be
collected last."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(cuda, seed, B, Hq, Hkv, L):
    g = torch.Generator(cuda).manual_seed(seed)
    q = torch.randn(B, Hq, 128, device=cuda, generator=g).bfloat16()
    kc = torch.randn(B, Hkv, L, 128, device=cuda, generator=g).bfloat16()
    vc = torch.randn(B, Hkv, L, 128, device=cuda, generator=g).bfloat16()
    return q, kc, vc


def _noalloc(vm, out, q, kc, vc, kv_len):
    lib = vm.lib()
    B, Hq, D = q.shape
    st = torch.cuda.current_stream().cuda_stream
    return lib.vmlx_cuda_sdpa_decode_noalloc(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, Hq,
                                             kc.shape[1], D, kv_len, kc.shape[2], D ** -0.5, st)


def _with_workspace(vm, q, kc, vc, kv_len):
    lib = vm.lib()
    B, Hq, D = q.shape
    nbytes = lib.vmlx_cuda_sdpa_decode_workspace(B, Hq, kv_len, D)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=q.device)  # split counters start at zero
    out = torch.empty_like(q)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.vmlx_cuda_sdpa_decode(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, Hq, kc.shape[1],
                                   D, kv_len, kc.shape[2], D ** -0.5, ws.data_ptr(), nbytes, st)
    assert rc == 0, lib.vmlx_last_error()
    return out


def test_noalloc_matches_workspace_version_twice(vm, cuda):
    for seed, (B, Hq, Hkv, L, kv_len) in enumerate([(2, 32, 8, 4200, 4097), (3, 8, 2, 700, 513)]):
        q, kc, vc = _inputs(cuda, 100 + seed, B, Hq, Hkv, L)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(vm, out, q, kc, vc, kv_len)
        assert rc == 0, vm.lib().vmlx_last_error()
        ref = _with_workspace(vm, q, kc, vc, kv_len)
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert torch.equal(out, ref)  # the same kernel on the same inputs: the same bits


def test_noalloc_rejects_sizes_beyond_scratch(vm, cuda):
    q, kc, vc = _inputs(cuda, 7, 1, 8, 8, 64)
    out = torch.empty_like(q)
    lib = vm.lib()
    st = torch.cuda.current_stream().cuda_stream
    # 256 sequences x 64 heads x 64 splits x 130 floats is far beyond 8 MiB
    rc = lib.vmlx_cuda_sdpa_decode_noalloc(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), 256, 64, 8,
                                           128, 16384, 16384, 0.088, st)
    assert rc == 1
    assert b"built-in scratch" in lib.vmlx_last_error()
