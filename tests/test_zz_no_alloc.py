"""finch_matvec_noalloc: the matvec for callers that may not allocate device memory.

Some callers of this library cannot call cudaMalloc at the point where they
need a matvec -- an engine that has given all of HBM to its own pool, a plugin
callback that runs under a "no allocation" rule, a thread that must not block
on the driver.  For them the library carries a fixed staging buffer inside its
own image and this entry point uses only that.  The test calls it through the C
ABI twice in a row (the second call reuses the buffer with the first call's
contents still in it) and checks each result against the regular entry point
and against the CPU oracle.
It is collected last so that a failure here cannot hide any other test.
"""
import ctypes as C

import numpy as np
import pytest

from finchmoe_b200 import lib as L
from finchmoe_b200 import synth
from oracle import oracle as orc
from parity import assert_close

pytestmark = pytest.mark.gpu


def test_matvec_noalloc_matches_regular_entry_point_twice():
    from finchmoe_b200 import api
    ctx = api.Context(hidden=256, n_experts=8, top_k=8, moe_inter=128, shared_inter=128, n_layers=1, max_tokens=1)
    try:
        so = ctx.lib
        rng = synth.rng_for(4, 321)
        cases = [(synth.affine_tensor(rng, 96, 2048, 3, L.FP16), 2), (synth.affine_tensor(rng, 64, 1024, 4, L.BF16), 5),
                 (synth.gguf_tensor(rng, 40, 512, 12), 1)]
        for rep in range(2):
            for t, M in cases:
                w = ctx.upload_tensor(t)
                x = np.ascontiguousarray(rng.normal(0, 1, size=(M, t["in_dim"])).astype(np.float32))
                want = ctx.fast_dequant_matvec(w, x)
                got = np.full((M, t["out_dim"]), np.nan, np.float32)
                rc = so.finch_matvec_noalloc(C.byref(w), x.ctypes.data, got.ctypes.data, M, None)
                assert rc == L.OK, rc
                # the regular entry point may pick a different kernel for the same tensor (streaming kernel for
                # few positions), so the two agree to the path's tolerance, not bit for bit
                assert_close(got, want, f"noalloc vs regular, rep {rep} bits={t['bits']}")
                # and, directly, against the CPU oracle
                ref = orc.matvec(t["W"], t.get("S"), t.get("B"), t.get("scale_dtype", L.FP16), x, t["out_dim"], t["in_dim"], t["group"],
                                 t["bits"], orc.ACC_F64)
                assert_close(got, ref, f"noalloc vs oracle, rep {rep} bits={t['bits']}")
        # a call that does not fit the fixed buffer is refused, not truncated
        big = synth.affine_tensor(rng, 64, 4096, 4, L.BF16)
        wb = ctx.upload_tensor(big)
        xb = np.zeros((40, 4096), np.float32)
        ob = np.zeros((40, 64), np.float32)
        assert so.finch_matvec_noalloc(C.byref(wb), xb.ctypes.data, ob.ctypes.data, 40, None) == L.E_UNSUPPORTED
        assert so.finch_matvec_noalloc(None, xb.ctypes.data, ob.ctypes.data, 1, None) == L.E_ARG
    finally:
        ctx.destroy()
