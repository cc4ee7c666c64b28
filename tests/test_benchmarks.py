"""Model benchmark suite: every model builds and trains in both arms at a
reduced scale on the CPU, the harness reports the reference's fields
(reference: benchmarks/src/harness.rs, tier1/*, tier2/*)."""
import pytest

from flodl_b200.benchmarks import SUITE, run_benchmark


@pytest.mark.parametrize("name", list(SUITE))
def test_suite_model_runs_both_arms(name):
    for arm in ("flodl", "torch"):
        r = run_benchmark(name, arm, "cpu", runs=2, warmup_epochs=1, measured_epochs=2,
                          batches_per_epoch=2, scale=0.0625, batch_scale=0.0625)
        assert len(r.epoch_times_ms) == 2 and r.median_epoch_ms > 0
        assert r.param_count > 0 and r.final_loss == r.final_loss  # finite, not NaN
        assert len(r.run_medians_ms) == 1
