"""Every example program runs on the CPU and learns (reference: the
flodl/examples programs, hf-ddp)."""
import pytest


def test_sine_wave():
    from flodl_b200.examples.sine_wave import run
    r = run(400)
    assert r["final_loss"] < 0.05 * r["first_loss"]


def test_mixed_precision():
    from flodl_b200.examples.mixed_precision import run
    r = run(150)
    assert r["final_loss"] < 0.3 * r["first_loss"] and r["weight_dtype"] == "torch.float32"


def test_transfer_learning():
    from flodl_b200.examples.transfer_learning import run
    r = run(150)
    assert r["loaded"] == 4 and r["encoder_unchanged"] and r["final_loss"] < r["first_loss"]


def test_observation():
    from flodl_b200.examples.observation import run
    r = run(40)
    assert r["epochs"] >= 8 and "hidden" in r["metrics"]


def test_flowbuilder_residual():
    from flodl_b200.examples.flowbuilder_residual import run
    r = run(150)
    assert r["final_loss"] < 0.5 * r["first_loss"] and "res2" in r["tags"]


def test_showcase():
    from flodl_b200.examples.showcase import run
    r = run(60)
    assert r["final_loss"] < r["first_loss"] and r["nodes"] >= 6 and r["svg"] > 100


def test_auto_promote_single_and_two_cpu_ranks():
    from flodl_b200.examples.auto_promote import run
    one = run(0, epochs=2)
    assert one["world"] == 1 and one["epoch_losses"][-1] < one["epoch_losses"][0]
    two = run(2, epochs=2)
    assert two["world"] == 2 and two["syncs"] > 0


@pytest.mark.parametrize("tier", ["managed", "cooperative"])
def test_hf_ddp_tiers(tier):
    from flodl_b200.examples.hf_ddp import run
    r = run(tier, epochs=3)
    assert r["last"] < r["first"]


def test_dnaseq_conv1d():
    from flodl_b200.examples.dnaseq_conv1d import run
    r = run(epochs=8, n_train=2000, n_val=300, L=64)  # shorter sequences than the default 200
    assert r["val_accuracy"] > 0.9


def test_dna_autoencoder():
    from flodl_b200.examples.dna_autoencoder import run
    r = run(epochs=25, n=256)
    assert r["per_base_accuracy"] > 0.5 and r["reload_matches"] and r["latent_shape"] == [2, 32]


def test_regression():
    from flodl_b200.examples.regression import run
    r = run()
    assert abs(r["slope"] - 2) < 0.05 and abs(r["intercept"] - 1) < 0.05
    assert r["logistic_accuracy"] > 0.95


def test_schedulers():
    from flodl_b200.examples.schedulers import run
    r = run()
    assert r["lr_peak"] <= 1e-3 + 1e-12 and r["lr_final"] < r["lr_peak"] and r["final_loss"] < r["first_loss"]
