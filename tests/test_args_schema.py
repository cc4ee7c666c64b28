"""Declarative arguments with --fdl-schema, the schema cache and `config show`
(reference: flodl-cli-macros/src/lib.rs, flodl-cli/src/args/, schema_cache.rs,
cli/schema.rs, cli/config.rs)."""
import json
import os
import subprocess
import sys
import textwrap
import time
from dataclasses import dataclass
from typing import List, Optional

import pytest

from flodl_b200.args import ArgsError, arg, option, parse_or_schema, schema_of, try_parse
from flodl_b200 import schema as sch
from flodl_b200.manifest import show_config

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@dataclass
class TrainArgs:
    """Train a model."""
    model: str = option("mlp", short="m", choices=["mlp", "resnet"], help="Model architecture.")
    epochs: int = option(10, short="e", help="Number of epochs.")
    lr: float = option(1e-3, help="Learning rate.")
    verbose: bool = option(False, short="v", help="Chatty output.")
    wandb_key: Optional[str] = option(None, env="FLODL_TEST_WANDB_KEY", help="API key.")
    tags: List[str] = option([], help="Repeatable tag.")
    datasets: List[str] = arg(variadic=True, help="Dataset paths.")


def test_parse_types_defaults_shorts_and_lists(monkeypatch):
    monkeypatch.delenv("FLODL_TEST_WANDB_KEY", raising=False)
    a = try_parse(TrainArgs, ["-m", "resnet", "--epochs=3", "-v", "--tags", "x", "--tags", "y",
                              "d1", "d2"])
    assert (a.model, a.epochs, a.lr, a.verbose, a.wandb_key) == ("resnet", 3, 1e-3, True, None)
    assert a.tags == ["x", "y"] and a.datasets == ["d1", "d2"]
    monkeypatch.setenv("FLODL_TEST_WANDB_KEY", "k")
    assert try_parse(TrainArgs, []).wandb_key == "k"


@pytest.mark.parametrize("argv,msg", [(["--model", "vit"], "not one of"),
                                       (["--epoch", "3"], "did you mean --epochs"),
                                       (["--lr", "fast"], "invalid float")])
def test_parse_errors(argv, msg):
    with pytest.raises(ArgsError, match=msg):
        try_parse(TrainArgs, argv)


def test_schema_shape_matches_the_reference_contract():
    s = schema_of(TrainArgs)
    assert s["args"] == [{"name": "datasets", "type": "list[string]", "description": "Dataset paths.",
                          "required": False, "variadic": True}]
    o = s["options"]
    assert o["model"] == {"type": "string", "description": "Model architecture.", "default": "mlp",
                          "choices": ["mlp", "resnet"], "short": "m"}
    assert o["epochs"]["type"] == "int" and o["lr"]["type"] == "float"
    assert o["verbose"]["type"] == "bool" and o["wandb-key"]["env"] == "FLODL_TEST_WANDB_KEY"
    assert o["tags"]["type"] == "list[string]"
    sch.check_schema(s)


def test_reserved_names_are_refused():
    @dataclass
    class Bad:
        help: bool = option(False)
    with pytest.raises(TypeError, match="reserved"):
        schema_of(Bad)


def test_parse_or_schema_intercepts(capsys):
    with pytest.raises(SystemExit) as e:
        parse_or_schema(TrainArgs, ["train", "--fdl-schema"])
    assert e.value.code == 0
    assert json.loads(capsys.readouterr().out)["options"]["epochs"]["default"] == 10
    with pytest.raises(SystemExit) as e:
        parse_or_schema(TrainArgs, ["train", "--nope"])
    assert e.value.code == 2


def _project(tmp_path):
    (tmp_path / "train.py").write_text(textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {ROOT!r})
        from dataclasses import dataclass
        from flodl_b200.args import option, parse_or_schema
        @dataclass
        class A:
            epochs: int = option(1, help="Epochs.")
            opt: str = option("sgd", choices=["sgd", "adam"], help="Optimizer.")
        a = parse_or_schema(A)
        print("epochs", a.epochs, a.opt)
        """))
    (tmp_path / "fdl.yml").write_text(textwrap.dedent(f"""
        commands:
          train:
            description: train
            run: {sys.executable} train.py
          hello: echo hello
        """))
    (tmp_path / "fdl.prod.yml").write_text("commands:\n  train:\n    description: prod train\n")
    return str(tmp_path)


def test_schema_cache_refresh_list_stale_orphan_clear(tmp_path):
    proj = _project(tmp_path)
    done = sch.refresh(proj)
    assert done == ["train"]  # `echo hello --fdl-schema` prints no JSON: skipped
    entries = {e.cmd_name: e.status for e in sch.discover(proj)}
    assert entries == {"train": "fresh"}
    cached = sch.load_cached(proj, "train")
    assert cached["options"]["opt"]["choices"] == ["sgd", "adam"]
    assert sch.validate_tail(cached, ["--epochs", "3", "--opt", "adam"]) == []
    errs = sch.validate_tail(cached, ["--epoch", "3", "--opt", "lamb"])
    assert "did you mean --epochs" in errs[0] and "not one of" in errs[1]
    # the script changed after the cache was written: stale
    later = time.time() + 5
    os.utime(os.path.join(proj, "train.py"), (later, later))
    assert {e.cmd_name: e.status for e in sch.discover(proj)} == {"train": "stale"}
    # the command left the manifest: orphan
    with open(os.path.join(proj, "fdl.yml"), "w") as f:
        f.write("commands:\n  hello: echo hello\n")
    assert {e.cmd_name: e.status for e in sch.discover(proj)} == {"train": "orphan"}
    assert sch.clear(proj) == 1 and sch.discover(proj) == []


def test_cli_schema_and_config_show(tmp_path):
    proj = _project(tmp_path)
    run = lambda *a: subprocess.run([sys.executable, "-m", "flodl_b200", *a], cwd=proj,
                                    capture_output=True, text=True,
                                    env=dict(os.environ, PYTHONPATH=ROOT))
    r = run("schema", "refresh", "train")
    assert r.returncode == 0 and "cached 1" in r.stdout, r.stderr
    r = run("schema", "list", "--json")
    assert json.loads(r.stdout)[0]["status"] == "fresh"
    # `run` checks the extra arguments against the cached schema
    r = run("run", "train", "--", "--opt", "lamb")
    assert r.returncode == 2 and "not one of" in r.stderr
    r = run("run", "train", "--", "--opt", "adam")
    assert r.returncode == 0 and "epochs 1 adam" in r.stdout
    lines = show_config(proj, "prod")
    desc = [l for l in lines if l.startswith("commands.train.description")][0]
    assert '"prod train"' in desc and desc.endswith("# fdl.prod.yml")
    r = run("config", "show")
    assert "commands.train.description" in r.stdout and "# fdl.yml" in r.stdout
