"""The routing plan's no-allocation entry point (dmoe_route_plan_noalloc), called through the
C ABI, against the regular entry point with a caller workspace (dmoe_route_plan).

It serves callers that cannot allocate device memory around a call (an FFI host that only
holds its input/output buffers, or a serving loop whose device memory belongs to another
allocator and where cudaMalloc/cudaFree may not run).  Its scratch is a library-owned static
device array shared by all calls, so two calls in a row must not see each other's state.
This file is collected last on purpose.
"""

import ctypes

import pytest
import torch

gpu = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _ptr(t):
    return None if t is None else t.data_ptr()


def _plan_outputs(T, k, E, wdt):
    return dict(counts=torch.full((E,), -1, dtype=torch.int32, device=DEV),
                offsets=torch.full((E + 1,), -1, dtype=torch.int32, device=DEV),
                perm_token=torch.full((T * k,), -1, dtype=torch.int32, device=DEV),
                perm_slot=torch.full((T * k,), -1, dtype=torch.int32, device=DEV),
                inverse=torch.full((T * k,), -1, dtype=torch.int32, device=DEV),
                perm_weight=torch.zeros(T * k, dtype=wdt, device=DEV))


def _call(lib, noalloc, idx, w, E):
    T, k = idx.shape
    out = _plan_outputs(T, k, E, w.dtype)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    common = (idx.data_ptr(), w.data_ptr(), 2, T, k, E, out["counts"].data_ptr(), out["offsets"].data_ptr(),
              out["perm_token"].data_ptr(), out["perm_slot"].data_ptr(), out["inverse"].data_ptr(),
              out["perm_weight"].data_ptr())
    if noalloc:
        rc = lib.dmoe_route_plan_noalloc(*common, stream)
    else:
        ws_bytes = lib.dmoe_route_plan_workspace_size(T, k, E)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        rc = lib.dmoe_route_plan(*common, ws.data_ptr(), ws_bytes, stream)
    assert rc == 0, lib.dmoe_last_error().decode()
    torch.cuda.synchronize(DEV)
    return out


def _routing(T, k, E, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g).to(torch.bfloat16)
    return idx.to(DEV), w.to(DEV)


@gpu
def test_noalloc_plan_matches_workspace_plan_twice_in_a_row():
    from distributedmoe_b200 import _native as N
    lib = N.lib()
    # Two different routings back to back: the second call reuses the shared static scratch.
    for T, k, E, seed in [(4096, 8, 256, 1), (3000, 2, 8, 2)]:
        idx, w = _routing(T, k, E, seed)
        mine = _call(lib, True, idx, w, E)
        ref = _call(lib, False, idx, w, E)
        for key in ref:
            assert torch.equal(mine[key], ref[key]), key  # integer work: bit-exact


@gpu
def test_noalloc_plan_rejects_sizes_beyond_its_static_scratch():
    from distributedmoe_b200 import _native as N
    lib = N.lib()
    T, k, E = 300000, 8, 1024  # needs ~4.6 MB of scratch, more than the 512 KiB array
    rc = lib.dmoe_route_plan_noalloc(None, None, 2, T, k, E, None, None, None, None, None, None, None)
    assert rc == 1
    assert b"static" in lib.dmoe_last_error()
