"""CSA2 cross-layer reuse (``linattn_b200.csa2_stack``) against the reference's
``CrossLayerPlan`` / ``CSA2Stack`` semantics (``tests/golden/csa2_stack.npz``): the plan,
the storage accounting, and the oracle layer run with the representatives' K / V
reproducing the reference stack's outputs.  CPU only."""

import numpy as np
import pytest

from oracle.csa2 import boundary_tied_rows, csa2_attend
from linattn_b200.core import AttnConfig
from linattn_b200.csa2_stack import (CrossLayerPlan, CSA2StackConfig, csa2_stack_bytes, csa2_stack_describe,
                                     share_layers)
from tests.conftest import golden

ATTN = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, seed=5)
CFG = CSA2StackConfig(n_layers=4, layer_group=2, compress_ratio=8, bits=4, topk_groups=3, window=24)


def test_plan():
    plan = CrossLayerPlan(n_layers=10, group_size=4)
    assert plan.groups == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    assert plan.stored_layers == [0, 4, 8] and plan.copies == 3
    assert plan.bytes_multiplier == pytest.approx(0.3)
    assert [plan.representative(i) for i in range(10)] == [0, 0, 0, 0, 4, 4, 4, 4, 8, 8]
    assert plan.is_full(4) and not plan.is_full(5)
    with pytest.raises(IndexError):
        plan.representative(10)
    with pytest.raises(ValueError):
        CrossLayerPlan(n_layers=0)
    stored, mapping = share_layers(list("abcdefghij"), plan)
    assert stored == {0: "a", 4: "e", 8: "i"} and mapping[9] == 8


def test_accounting_against_reference():
    g = golden("csa2_stack")
    assert csa2_stack_bytes(CFG, ATTN, 96, 4) / 96 == pytest.approx(float(g["bytes_per_token"]))
    assert csa2_stack_describe(CFG, ATTN) == str(g["spec"])
    unshared = CSA2StackConfig(**{**CFG.__dict__, "share": False})
    assert csa2_stack_bytes(unshared, ATTN, 96, 4) / 96 == pytest.approx(float(g["cmp_bytes_per_token_unshared"]))
    assert CrossLayerPlan(4, 2).copies == int(g["copies"])


def test_oracle_stack_against_reference():
    g = golden("csa2_stack")
    q, k, v = g["q"], g["k"], g["v"]
    plan = CrossLayerPlan(4, 2)
    for layer in range(4):
        src = plan.representative(layer)
        out, _ = csa2_attend(q[layer], k[src], v[src], np.asarray(_q_proj()), np.full(4, 0.25, np.float32),
                             ratio=8, bits=4, group=32, window=24, topk_groups=3)
        tied = boundary_tied_rows(g[f"scores_l{layer}"][0], ratio=8, window=24, topk_groups=3, chunk=96)
        err = np.abs(out - g["out"][layer])[0].max(-1)
        assert err[~tied].max() < 2e-5, layer


def _q_proj():
    from linattn_b200.csa2 import CudaCSA2Attention

    return CudaCSA2Attention(ATTN.with_(extras={"compress_ratio": 8})).q_proj.detach().numpy()
