"""RMSNorm after the assembly (``dwa_rmsnorm_fwd`` / ``dwa_rmsnorm_bwd``) against
the oracle in float64: f32 and bf16 inputs, f32 and bf16 outputs, the
assembly's shape (B*T rows of d_B = 1024) and a ragged row count; gradients
through ``torch.autograd`` (``rms_norm``) for x and scale."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from matrix_b200.synthetic import bf16_round
from oracle import dwa_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,d,x_dt,y_dt", [
    (4096, 1024, torch.bfloat16, torch.float32),
    (4096, 1024, torch.bfloat16, torch.bfloat16),
    (1003, 264, torch.float32, torch.float32),
    (37, 2048, torch.float32, torch.bfloat16),
])
def test_rms_norm_matches_oracle(rows, d, x_dt, y_dt):
    from matrix_b200.norm import rms_norm
    rng = np.random.default_rng(rows + d)
    x = rng.standard_normal((rows, d), dtype=np.float32) * np.float32(3.0)
    g = rng.standard_normal((rows, d), dtype=np.float32)
    scale = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    if x_dt == torch.bfloat16:
        x = bf16_round(x)
    if y_dt == torch.bfloat16:
        g = bf16_round(g)
    xt = torch.from_numpy(x).cuda().to(x_dt).requires_grad_(True)
    st = torch.from_numpy(scale).cuda().requires_grad_(True)
    y = rms_norm(xt, st, 1e-6, y_dt)
    assert y.dtype == y_dt and y.shape == (rows, d)
    y.backward(torch.from_numpy(g).cuda().to(y_dt))
    torch.cuda.synchronize()
    f = np.float64
    ry = O.rms_norm(x.astype(f), scale.astype(f))
    rgx, rgs = O.rms_norm_bwd(x.astype(f), scale.astype(f), g.astype(f))
    tol_y = 1e-5 if y_dt == torch.float32 else 1e-2
    tol_gx = 1e-5 if x_dt == torch.float32 else 1e-2
    assert_close(y.detach().float().cpu().numpy(), ry, tol_y, name="y")
    assert_close(xt.grad.float().cpu().numpy(), rgx, tol_gx, name="g_x")
    assert_close(st.grad.cpu().numpy(), rgs, 1e-5, name="g_scale")
    assert xt.grad.dtype == x_dt


def test_module_default_is_identity_scale_and_deterministic():
    from matrix_b200.norm import RMSNorm
    m = RMSNorm(1024, device="cuda")
    x = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = m(x)
    ms = (y.double() ** 2).mean(dim=1)
    assert torch.allclose(ms, torch.ones_like(ms), rtol=1e-4)
    g = torch.randn_like(y)
    grads = []
    for _ in range(2):
        x.grad = None
        m.scale.grad = None
        m(x).backward(g)
        grads.append((x.grad.clone(), m.scale.grad.clone()))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])
