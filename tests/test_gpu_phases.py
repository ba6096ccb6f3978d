"""Per-phase device timing (yabt_b200.phases, C ABI yabt_phase_*) (GPU tests):
every launch group of a boosting iteration is recorded under its phase, and
host-issued work can be bracketed as a phase of its own."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_phases_of_a_boosting_iteration():
    from yabt_b200 import Booster, BoostParams, MSELoss, phases
    rng = np.random.default_rng(3)
    X = rng.normal(size=(20000, 12)).astype(np.float32)
    y = (X[:, 0] + X[:, 1] * X[:, 2]).astype(np.float32)
    assert phases.names()[:4] == ["begin", "hist", "reduce", "exchange"]
    phases.start(4096)
    Booster(BoostParams(n_estimators=2, max_leaves=31), MSELoss()).fit(X, y)
    torch.cuda.synchronize()
    rec = phases.read()
    phases.stop()
    for name in ("binning", "begin", "hist", "reduce", "scan", "finalize", "partition", "plan", "finish",
                 "leafnet", "interaction", "update"):
        assert rec.get(name, {}).get("ranges", 0) > 0, (name, rec)
        assert rec[name]["ms"] >= 0.0
    assert "exchange" not in rec                    # one GPU: no cross-GPU exchange
    # a stopped recorder records nothing more; start() clears earlier ranges
    Booster(BoostParams(n_estimators=1, max_leaves=31), MSELoss()).fit(X, y)
    assert phases.read() == rec
    phases.start(16)
    with phases.host_phase():
        torch.ones(1 << 20, device="cuda").sum()
    torch.cuda.synchronize()
    assert phases.read()["collective"]["ranges"] == 1
    phases.stop()
