"""The failure path of the kernels' bounded waits, exercised without a fault.

``kda_selftest_wait_timeout`` runs the mbarrier wait every kernel uses on a
barrier that nothing completes; the wait gives up after a few thousand polls
(well under a millisecond), the CTA records it and returns.  The host reads it
through ``kda_device_status``; the context stays usable (a forward afterwards
matches the oracle) and clearing resets the flags.
"""

import numpy as np
import pytest
import torch

from oracle import kda_oracle as K

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_reports_and_the_context_survives():
    import axiom_b200 as A
    from axiom_b200._lib import KDAError

    A.device_status(clear=True)
    assert not any(A.device_status().values())
    A.selftest_wait_timeout(4096)
    st = A.device_status()
    assert st["selftest"] and not (st["fwd"] or st["bwd"] or st["decode_fused"])
    with pytest.raises(KDAError) as e:
        A.check_device(clear=True)
    assert e.value.status == -9
    assert not any(A.device_status().values())
    # the context still runs kernels correctly
    x = K.make_inputs(1, 200, 2, 128, 128, seed=9, s0_std=0.05)
    xr = {k: (K.bf16_round(v) if k != "S0" else v) for k, v in x.items()}
    dev = {k: torch.as_tensor(np.ascontiguousarray(v), dtype=torch.float32).cuda()
           .to(torch.bfloat16 if k != "S0" else torch.float32).contiguous() for k, v in x.items()}
    o, s_t, _ = A.kda_fwd(dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"], dev["S0"], o_dtype=torch.float32)
    o_ref, s_ref = K.chunk_fwd(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], xr["S0"], chunk=64)
    assert K.scale_rel_err(o.cpu().numpy(), o_ref) <= 1e-2
    assert K.scale_rel_err(s_t.cpu().numpy(), s_ref) <= 1e-2
    A.check_device()  # no kernel gave up
