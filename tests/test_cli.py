"""Command line: probe, diagnose, status/start against a live status board,
init scaffold, completions (reference: flodl-cli/src/cli_tests.rs)."""
import json
import subprocess
import sys

from flodl_b200.cli import diagnose_checks, main
from flodl_b200.parallel.membership import StartMode
from flodl_b200.parallel.portmux import PortMux, StatusBoard


def test_probe_json_with_spoofed_hardware(monkeypatch, capsys):
    monkeypatch.setenv("FLODL_TESTING_GPU_JSON", json.dumps([{"arch": "10.0", "name": "NVIDIA B200"}] * 2))
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    assert main(["probe", "--json"]) == 0
    r = json.loads(capsys.readouterr().out)
    assert [g["arch"] for g in r["gpus"]] == ["sm_100", "sm_100"] and r["cpus"] > 0


def test_diagnose_flags_uncovered_arch(monkeypatch):
    monkeypatch.setenv("FLODL_TESTING_GPU_JSON", json.dumps([{"arch": "9.0"}]))
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    rows = {c: s for c, s, _ in diagnose_checks()}
    assert rows["native runtime (_native)"] == "OK" and rows["GPU 0 arch"] == "FAIL"
    assert main(["diagnose"]) == 1


def test_status_and_start(capsys):
    mux = PortMux()
    board = StatusBoard()
    mux.serve_status(board)
    hp = f"127.0.0.1:{mux.port}"
    assert main(["status", hp]) == 1  # nothing published yet
    capsys.readouterr()
    board.publish({"phase": "joining", "members": 1})
    assert main(["status", hp, "--json"]) == 0
    st = json.loads(capsys.readouterr().out)
    assert st["phase"] == "joining" and st["members"] == 1
    board.configure_start(StartMode.Manual, "ff" * 16)
    assert main(["start", hp]) == 0 and board.start_requested()
    mux.close()


def test_init_scaffold_runs(tmp_path):
    d = tmp_path / "proj"
    assert main(["init", str(d)]) == 0
    assert main(["init", str(d)]) == 1  # refuses to overwrite
    r = subprocess.run([sys.executable, "-c",
                        f"import runpy; m = runpy.run_path({str(d / 'train.py')!r}); m['main'](51)"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "step 50 loss" in r.stdout


def test_completions(capsys):
    assert main(["completions", "bash"]) == 0
    assert "complete -F _flodl_b200" in capsys.readouterr().out


def test_manifest_overlays_and_run(tmp_path, monkeypatch, capsys):
    from flodl_b200.manifest import deep_merge, load_manifest, resolve
    (tmp_path / "fdl.yml").write_text(
        "env: {A: '1'}\ncommands:\n  hello: {run: 'echo hello', append: '--x'}\n  gone: {run: 'true'}\n  sub:\n")
    (tmp_path / "fdl.ci.yml").write_text("commands:\n  hello: {append: '--ci'}\n  gone:\n")
    (tmp_path / "sub").mkdir()
    (tmp_path / "sub" / "fdl.yml").write_text("commands:\n  inner: {run: 'echo inner'}\n")
    assert deep_merge({"a": {"b": 1, "c": 2}}, {"a": {"c": None, "d": 3}}) == {"a": {"b": 1, "d": 3}}
    m = load_manifest(str(tmp_path), "ci")
    assert m["commands"]["hello"]["append"] == "--ci" and "gone" not in m["commands"]
    spec, d = resolve(m, "sub:inner", str(tmp_path))
    assert spec["run"] == "echo inner" and d.endswith("sub")
    monkeypatch.chdir(tmp_path)
    assert main(["run", "--dry-run", "hello", "@ci", "--", "extra"]) == 0
    assert capsys.readouterr().out.strip() == "echo hello --ci extra"
    assert main(["run", "sub:inner"]) == 0
    assert main(["commands", "@ci"]) == 0
    out = capsys.readouterr().out
    assert "hello" in out and "sub-manifest" in out and "gone" not in out


def test_repo_manifest_parses():
    import os
    from flodl_b200.manifest import list_commands
    root = os.path.dirname(os.path.dirname(__file__))
    cmds = list_commands(root, "quick")
    assert {"build", "test", "test-gpu", "bench"} <= set(cmds)


def test_api_ref_add_hf_and_publish(tmp_path, capsys):
    from flodl_b200.cli import api_reference, publish
    ref = api_reference("flodl_b200.parallel")
    assert "ChunkPool" in ref["flodl_b200.parallel.coordinator"]
    assert main(["add", "hf", "--dir", str(tmp_path)]) == 0
    assert (tmp_path / "flodl-hf" / "main.py").exists()
    assert "flodl-hf:" in (tmp_path / "fdl.yml").read_text()
    compile((tmp_path / "flodl-hf" / "main.py").read_text(), "main.py", "exec")
    src = tmp_path / "job"
    src.mkdir()
    (src / "train.py").write_text("print('hi')\n")
    man = publish(str(src), str(tmp_path / "pub"))
    assert man["files"] == ["train.py"] and (tmp_path / "pub" / man["run"] / "train.py").exists()
    (src / "bad.py").write_text("def x(:\n")
    assert main(["publish", str(src), str(tmp_path / "pub")]) == 1
