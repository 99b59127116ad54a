"""The allocation-free router entry point against the workspace router.

moe_route_tokens_noalloc serves callers that cannot allocate device memory (a host binding with
no CUDA allocator of its own, code running under stream capture, an embedding with a fixed
device-memory budget): it keeps the router's workspace in a static device array instead of taking
one from the caller. Its results must equal moe_route_tokens' on the same inputs, call after call,
although the static array keeps whatever the previous call left in it.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _bf16(rng, shape, std):
    return torch.from_numpy((rng.normal(0, std, shape)).astype(np.float32)).to(torch.bfloat16).cuda()


def _noalloc(L, x, w, bias, k, mode, n_group, topk_group, scale):
    T, H = x.shape
    E = w.shape[0]
    ids = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    wt = torch.full((T, k), float("nan"), dtype=torch.float32, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.moe_route_tokens_noalloc(x.data_ptr(), w.data_ptr(), 0 if bias is None else bias.data_ptr(), T, H, E, k,
                                    mode, n_group, topk_group, scale, ids.data_ptr(), wt.data_ptr(), st)
    return rc, ids, wt


def test_noalloc_router_matches_workspace_router_on_consecutive_calls():
    from moe_b200 import _lib, route_tokens

    L = _lib.lib()
    rng = np.random.default_rng(11)
    cases = [
        # (T, H, E, k, mode, n_group, topk_group, scale): decode-sized renormalised softmax, then a
        # larger sigmoid-group call whose counters sit elsewhere in the array
        (64, 2048, 128, 8, _lib.ROUTER_SOFTMAX_RENORM, 1, 1, 1.0),
        (300, 1024, 64, 6, _lib.ROUTER_SIGMOID_GROUP, 8, 4, 2.5),
        (1, 2048, 128, 8, _lib.ROUTER_SOFTMAX_RENORM, 1, 1, 1.0),
    ]
    for T, H, E, k, mode, G, TG, scale in cases:
        x = _bf16(rng, (T, H), 1.0)
        w = _bf16(rng, (E, H), 0.02)
        bias = torch.from_numpy(rng.normal(0, 0.05, E).astype(np.float32)).cuda() if mode == 2 else None
        want_ids, want_w = route_tokens(x, w, k, mode, bias=bias, n_group=G, topk_group=TG, routed_scale=scale)
        rc, ids, wt = _noalloc(L, x, w, bias, k, mode, G, TG, scale)
        assert rc == _lib.MOE_OK, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, want_ids)
        # the routers share one kernel: weights agree bit for bit (the tolerance the router tests use)
        assert torch.equal(wt, want_w)


def test_noalloc_router_rejects_calls_beyond_its_array():
    from moe_b200 import _lib

    L = _lib.lib()
    T, E = 4096, 128  # needs about 2 MB of logits, the array holds 1 MiB
    assert L.moe_route_workspace_bytes(T, E) > (1 << 20)
    rc = L.moe_route_tokens_noalloc(None, None, None, T, 2048, E, 8, 1, 1, 1, 1.0, None, None, None)
    assert rc == _lib.MOE_ERR_INVALID
    assert "static scratch" in _lib.last_error()
