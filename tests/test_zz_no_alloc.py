"""avq_quantize_noalloc against avq_quantize, through the C ABI.

The entry point runs the quantizer kernels with their scratch in a fixed
device array instead of a caller workspace.  Both entry points launch the same
kernels on the same inputs, so the outputs must agree exactly (tolerance 0 for
the integer assignments and counts and for the narrowed and fp32 bucket sums).
Two calls in a row with different key counts check that nothing left in the
array by the first call leaks into the second.  The file is named to be
collected last, so it also runs after every other GPU test has used the
library on the same device.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from avqa_b200 import _lib, ops
from avqa_b200.codebook import codebook_from_keys

SCRATCH_BYTES = 16 << 20  # AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES in include/avqa_b200.h


def _noalloc(keys: torch.Tensor, values: torch.Tensor, cb: ops.PreparedCodebook) -> ops.QuantState:
    lib = _lib.load()
    B, H, S, D = keys.shape
    _, M0, C, _ = cb.dims
    G, dev, dt = B * H, keys.device, keys.dtype
    i32 = dict(dtype=torch.int32, device=dev)
    st = ops.QuantState(
        B, H, S, dt, torch.empty(G, S, **i32), torch.empty(G, S, **i32),
        torch.empty(G, M0, D, dtype=dt, device=dev), torch.empty(G, M0, C, D, dtype=dt, device=dev),
        torch.empty(G, M0, D, dtype=torch.float32, device=dev),
        torch.empty(G, M0, C, D, dtype=torch.float32, device=dev),
        torch.empty(G, M0, **i32), torch.empty(G, M0, C, **i32), torch.empty(G, **i32),
        torch.full((1,), 2 ** 31 - 1, **i32))
    rc = lib.avq_quantize_noalloc(_lib.dtype_code(dt), keys.data_ptr(), _lib.strides3(keys), values.data_ptr(),
                                  _lib.strides3(values), B, H, S, D, M0, C, cb.parents.data_ptr(),
                                  cb.p_sq.data_ptr(), cb.children.data_ptr(), cb.c_sq.data_ptr(),
                                  st.passign.data_ptr(), st.cassign.data_ptr(), st.pagg.data_ptr(),
                                  st.cagg.data_ptr(), st.pacc.data_ptr(), st.cacc.data_ptr(), st.pcnt.data_ptr(),
                                  st.ccnt.data_ptr(), st.nvalid.data_ptr(), st.gmin.data_ptr(),
                                  _lib.stream_of(dev))
    _lib.check(rc, "avq_quantize_noalloc")
    return st


def _inputs(seed: int, B: int, H: int, S: int, D: int, dtype: torch.dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(B, S, H * D, generator=g, device="cuda").to(dtype)
    v = torch.randn(B, S, H * D, generator=g, device="cuda").to(dtype)
    # module layout [B, S, H*D] viewed as [B, H, S, D], as the attention module passes it
    return k.view(B, S, H, D).transpose(1, 2), v.view(B, S, H, D).transpose(1, 2)


def test_oversized_request_is_rejected_before_touching_a_device() -> None:
    lib = _lib.load()
    B, H, S, M0 = 4, 32, 32768, 512
    need = lib.avq_quantize_workspace_size(B, H, S, M0)
    assert need > SCRATCH_BYTES
    s = (ctypes.c_longlong * 3)(1, 1, 1)
    rc = lib.avq_quantize_noalloc(1, None, s, None, s, B, H, S, 128, M0, 4, None, None, None, None, None, None,
                                  None, None, None, None, None, None, None, None, None)
    assert rc == 4  # AVQ_ERR_WORKSPACE
    msg = _lib.last_error()
    assert msg.startswith("avq_quantize_noalloc") and str(need) in msg and "avq_quantize with a workspace" in msg


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_noalloc_matches_workspace_entry_point_twice(dtype: torch.dtype) -> None:
    H, D, M0, C = 8, 128, 256, 4
    cases = [(1, 2, 4096), (2, 3, 1000)]  # (seed, B, S): the second call has fewer, differently sorted keys
    k0, _ = _inputs(99, 1, H, 2048, D, dtype)
    cbf = codebook_from_keys(k0[0].float(), M0, C, seed=3)
    cb = ops.prepare_codebook(cbf.parents, cbf.children, dtype, torch.device("cuda"))
    lib = _lib.load()
    for seed, B, S in cases:
        assert lib.avq_quantize_workspace_size(B, H, S, M0) <= SCRATCH_BYTES
        k, v = _inputs(seed, B, H, S, D, dtype)
        want = ops.quantize(k, v, cb, keep_sums=True)
        got = _noalloc(k, v, cb)
        torch.cuda.synchronize()
        for name in ("passign", "cassign", "pcnt", "ccnt", "nvalid", "gmin", "pacc", "cacc"):
            torch.testing.assert_close(getattr(got, name), getattr(want, name), rtol=0, atol=0, msg=name)
        for name in ("pagg", "cagg"):
            assert torch.equal(getattr(got, name).view(torch.int16), getattr(want, name).view(torch.int16)), name
