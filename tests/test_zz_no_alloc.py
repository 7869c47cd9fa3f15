"""The allocation-free decode entry point, for callers that cannot allocate device memory
(a plugin host or FFI binding that only hands over input and output buffers, or a process
that forbids device allocation after start-up).

It must give the same answer as the workspace entry point, on consecutive calls that reuse
the library's shared scratch, and reject shapes whose scratch need exceeds its 4 MiB.
Collected last (file name) so a failure here cannot stop the other GPU tests.
"""
import pytest
import torch

import oracle as O
from fnx import synth

pytestmark = pytest.mark.gpu


def test_decode_noalloc_matches_workspace_entry_point():
    from fnx import _lib
    from fnx.engine import MoELayer
    lib = _lib.lib()
    dev = torch.device("cuda")
    shape = synth.CFG2
    layer = MoELayer.from_synth(synth.make_layer(shape, seed=21, device=dev), shape)
    for call, M in enumerate((4, 1)):
        x = synth.make_tokens(M, shape.H, seed=40 + call, device=dev)
        ref_out, ref_w, ref_idx = layer.decode(x)
        out = torch.full_like(ref_out, float("nan"))
        w = torch.empty_like(ref_w)
        idx = torch.empty_like(ref_idx)
        rc = lib.fnx_moe_decode_w4_noalloc(
            x.data_ptr(), layer.router_cat.data_ptr(), layer.gu_t.data_ptr(), layer.dn_t.data_ptr(),
            layer.sh_gu_t.data_ptr(), layer.sh_dn_t.data_ptr(), None, out.data_ptr(), w.data_ptr(), idx.data_ptr(),
            M, shape.H, shape.I, shape.E, shape.k, _lib.stream(dev))
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx)
        assert torch.equal(w.view(torch.int16), ref_w.view(torch.int16))
        assert O.within_tolerance(out.cpu(), ref_out.cpu()), O.tolerance_report(out.cpu(), ref_out.cpu())
    assert _lib.device_errors() == 0
    # a shape whose scratch exceeds the static array is rejected before any launch
    big = lib.fnx_moe_decode_workspace(16, 8192, 4096, 2048, 32)
    assert big > 4 << 20
    rc = lib.fnx_moe_decode_w4_noalloc(*([None] * 10), 16, 8192, 4096, 2048, 32, None)
    assert rc == -5
