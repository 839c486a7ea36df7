"""CPU: the bf16-rounding restatement (oracle/bf16_math.py) used by the bf16
precision mode's parity test.

* rbf16 is round-to-nearest-even to bf16 (ties to even, carries into the
  exponent, signed zeros and infinities kept).
* With the rounding switched off, the restatement is the reference layer of
  ref_math.py: same outputs and gradients in fp64, for layers with and
  without node input -- so the bf16 oracle differs from the pinned one only
  at its rounding points.
"""
import copy

import numpy as np
import pytest
import torch

from conftest import small_graph


def test_rbf16_is_round_to_nearest_even():
    from oracle.bf16_math import rbf16
    one = 1.0
    ulp = 2.0 ** -7                     # bf16 spacing in [1, 2)
    x = torch.tensor([one + ulp / 2, one + 3 * ulp / 2, one + ulp / 2 + 2 ** -20, -(one + ulp / 2), 1.99999,
                      0.0, -0.0, float("inf"), 3.0e38], dtype=torch.float64)
    y = rbf16(x)
    assert y[0] == one                  # tie -> even mantissa
    assert y[1] == one + 2 * ulp        # tie -> even mantissa (up)
    assert y[2] == one + ulp            # above the tie -> up
    assert y[3] == -one
    assert y[4] == 2.0                  # carry into the exponent
    assert y[5] == 0 and torch.signbit(y[6]) and torch.isinf(y[7])
    assert torch.isfinite(y[8])


@pytest.mark.parametrize("dn,de", [(20, 12), (0, 16)])
def test_bf16_restatement_without_rounding_is_the_reference_layer(monkeypatch, dn, de):
    from fast_b200.model import GeneralModel
    from oracle import bf16_math, ref_math
    from oracle.sampler import OracleSampler
    g = small_graph(n_nodes=100, n_edges=5000, seed=2, int_ts=False, t_max=2e4, zipf=1.0)
    torch.manual_seed(1)
    nf = torch.randn(100, dn).double() if dn else None
    ef = torch.randn(5000, de).double()
    sp = dict(layer=2, neighbor=[5, 5], strategy="recent", prop_time=False, history=1, duration=0)
    gnn = dict(arch="transformer_attention", layer=2, att_head=2, dim_time=100, dim_out=100)
    m = GeneralModel(dn, de, sp, dict(type="none", dim_out=0), gnn,
                     dict(lr=1e-4, dropout=0.0, att_dropout=0.0)).double()
    m2 = copy.deepcopy(m)
    ora = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, 2, [5, 5], True, False, 1, 0.0)
    roots = np.concatenate([g["src"][3000:3050], g["dst"][3000:3050], g["src"][100:150]]).astype(np.int32)
    rts = np.concatenate([g["t"][3000:3050]] * 3).astype(np.float32)
    ora.sample(roots, rts)
    monkeypatch.setattr(bf16_math, "rbf16", lambda x: x)
    a = ref_math.model_forward(m, ora.get_ret(), nf, ef)
    b = ref_math.model_forward(m2, ora.get_ret(), nf, ef, layer_fn=bf16_math.layer_forward_bf16)
    la, lb = ref_math.bce_loss(*a), ref_math.bce_loss(*b)
    la.backward()
    lb.backward()
    assert torch.allclose(la, lb, rtol=1e-12, atol=0)
    for (n, p), q in zip(m.named_parameters(), m2.parameters()):
        assert torch.allclose(p.grad, q.grad, rtol=1e-9, atol=1e-15), n
