"""Plans (insight_b200_plan_create / _execute / _destroy): one spectral call
captured into a CUDA graph and replayed.

A plan's run must give exactly what the regular call gives on the same
tensors (the graph holds the same kernel launches), must pick up new input
contents written in place between runs, and must refuse host arrays.
"""
import numpy as np
import pytest

import insight_b200 as ib
from oracle import spectral_oracle as so

pytestmark = pytest.mark.gpu


def test_plan_welch_matches_the_call_and_follows_the_input(cuda):
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(21)
    x = torch.randn((1, 1 << 20), generator=g, device=cuda)
    kw = dict(fs=1e4, nperseg=1024, noverlap=512)
    ref = torch.empty((1, 513), dtype=torch.float64, device=cuda)
    ib.spectral(ib.OP_WELCH, x, out=ref, **kw)
    out = torch.full((1, 513), float("nan"), dtype=torch.float64, device=cuda)
    plan = ib.SpectralPlan(ib.OP_WELCH, x, out=out, **kw)
    n0 = ib.launch_count()
    plan.run(sync=True)
    assert ib.launch_count() - n0 == 1  # one graph launch
    assert torch.equal(out, ref)
    # new contents of x, same tensor: the next run follows them
    x.mul_(3.0)
    for _ in range(3):
        plan.run()
    torch.cuda.synchronize()
    _, r = so.welch(x[0].cpu().numpy(), **kw)
    assert so.max_rel_err(out[0].cpu().numpy(), r) <= 1e-5
    plan.close()


def test_plan_csd_transposed_and_stft(cuda):
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(22)
    X = torch.randn((3, 1 << 16), generator=g, device=cuda)
    Y = torch.randn((3, 1 << 16), generator=g, device=cuda)
    xt, yt = X.t(), Y.t()
    pc = torch.empty((3, 1025), dtype=torch.complex64, device=cuda)
    plan = ib.SpectralPlan(ib.OP_CSD, xt, yt, out=pc, axis=0, nperseg=2048)
    plan.run(sync=True)
    _, ref = ib.spectral(ib.OP_CSD, xt, yt, axis=0, nperseg=2048,
                         complex_output=True)
    assert torch.equal(pc, ref)
    plan.close()

    L, H = 2048, 512
    S = ((1 << 16) - L) // H + 1
    z = torch.empty((3, L // 2 + 1, S), dtype=torch.complex64, device=cuda)
    plan = ib.SpectralPlan(ib.OP_STFT, X, out=z, nperseg=L, noverlap=L - H)
    plan.run(sync=True)
    _, _, zr = so.stft(X[1].cpu().numpy(), nperseg=L, noverlap=L - H,
                       complex_output=True)
    assert so.max_rel_err(z[1].cpu().numpy(), zr) <= 1e-5
    plan.close()


def test_plan_refuses_host_arrays(cuda):
    x = np.zeros(4096, np.float32)
    out = np.zeros(129, np.float64)
    with pytest.raises(RuntimeError, match="GPU arrays"):
        ib.SpectralPlan(ib.OP_WELCH, x, out=out, nperseg=256)
