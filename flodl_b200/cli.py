"""Command line: ``python -m flodl_b200 <command>``.

Reference role: flodl-cli (``fdl``) - probe, diagnose, status, start, launch,
scaffold and shell completions (flodl-cli/src/{probe,diagnose.rs,status.rs,
init.rs,completions}). Build and download commands of the reference (libtorch,
NCCL) have no counterpart: this framework builds against the installed
PyTorch with ``python setup.py build_ext --inplace``.

Commands:

    probe [--json]                     GPUs, findings, driver, host memory
    diagnose [--json]                  import/extension/device/NCCL/peer checks
    status HOST:PORT [--json]          the controller's state.json
    start HOST:PORT [--token HEX]      arm a manual/hybrid start
    launch --devices D0,D1 [--policy abort|shrink] -- CMD ...
    init NAME                          scaffold a training script
    completions bash                   bash completion script
    commands [@env]                    commands of ./fdl.yml (with an overlay)
    run CMD [@env] [-- ARGS]           run a manifest command
    join HOST:PORT [--key-hex K]       dial a controller as this host's agent
    api-ref [MODULE] [--json]          public API surface with one-line docs
    add hf [--dir D]                   scaffold a HuggingFace playground + fdl.yml entry
    publish SRC DEST                   validate a run directory and publish its manifest
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import urllib.error
import urllib.request
from typing import List, Tuple

COMMANDS = ("probe", "diagnose", "status", "start", "launch", "init", "completions", "commands", "run",
            "join", "api-ref", "add", "publish")


def _probe(a) -> int:
    from .utils import hw
    r = hw.report()
    if a.json:
        print(json.dumps(r, indent=2))
        return 0
    print(f"driver {r['driver'] or 'n/a'}; host RAM {r['host_memory_mb'] / 1024:.0f} GiB "
          f"({r['host_available_mb'] / 1024:.0f} available); {r['cpus']} CPUs")
    if not r["gpus"]:
        print("no visible GPU")
    for g in r["gpus"]:
        print(f"  [{g['index']}] {g['name']}  {g['arch']}  {g['vram_mb'] / 1024:.0f} GiB")
    for n in r["notes"]:
        print(f"  note ({n['vendor']}, {n['kind']}): {n['message']}")
    return 0


def diagnose_checks() -> List[Tuple[str, str, str]]:
    """(check, OK|WARN|FAIL, detail) rows; read-only, changes no device setting."""
    rows = []
    try:
        import torch
        rows.append(("torch", "OK", f"{torch.__version__} (CUDA {torch.version.cuda})"))
    except Exception as e:
        return [("torch", "FAIL", repr(e))]
    from . import _ext
    rows.append(("native runtime (_native)", "OK" if _ext._native else "FAIL",
                 "loaded" if _ext._native else repr(_ext._NATIVE_ERR)))
    have_cuda = torch.cuda.is_available()
    c_state = "OK" if _ext._C else ("FAIL" if have_cuda else "WARN")
    rows.append(("sm_100a kernels (_C)", c_state, "loaded" if _ext._C else repr(_ext._C_ERR)))
    from .utils import hw
    gpus = hw.detect_gpus()
    if not gpus:
        rows.append(("GPUs", "WARN", "none visible: CPU paths only"))
    for g in gpus:
        ok = g.covered_by("10.0")
        rows.append((f"GPU {g.index} arch", "OK" if ok else "FAIL",
                     f"{g.name} {g.arch}" + ("" if ok else ": kernels are built for sm_100a only")))
    if have_cuda:
        try:
            v = torch.cuda.nccl.version()
            rows.append(("NCCL", "OK", ".".join(map(str, v)) if isinstance(v, tuple) else str(v)))
        except Exception as e:
            rows.append(("NCCL", "WARN", repr(e)))
        n = torch.cuda.device_count()
        missing = [(i, j) for i in range(n) for j in range(n)
                   if i != j and not torch.cuda.can_device_access_peer(i, j)]
        if n > 1:
            rows.append(("peer access", "OK" if not missing else "WARN",
                         f"all {n * (n - 1)} pairs" if not missing else f"no access for {missing[:4]}"))
    for k in ("NCCL_P2P_DISABLE", "NCCL_SHM_DISABLE", "NCCL_NVLS_ENABLE"):
        if k in os.environ:
            rows.append((k, "WARN", f"set to {os.environ[k]!r}"))
    return rows


def _diagnose(a) -> int:
    rows = diagnose_checks()
    if a.json:
        print(json.dumps([{"check": c, "state": s, "detail": d} for c, s, d in rows], indent=2))
    else:
        for c, s, d in rows:
            print(f"{s:5s} {c}: {d}")
    return 1 if any(s == "FAIL" for _, s, _ in rows) else 0


def _url(hostport: str, path: str) -> str:
    return f"http://{hostport}{path}"


def _status(a) -> int:
    try:
        body = urllib.request.urlopen(_url(a.controller, "/state.json"), timeout=10).read()
    except urllib.error.HTTPError as e:
        print(f"controller answered {e.code}: {e.read().decode(errors='replace')}", file=sys.stderr)
        return 1
    except OSError as e:
        print(f"controller unreachable: {e}", file=sys.stderr)
        return 1
    st = json.loads(body)
    if a.json:
        print(json.dumps(st, indent=2))
    else:
        for k, v in st.items():
            print(f"{k}: {v}")
    return 0


def _start(a) -> int:
    q = f"?token={a.token}" if a.token else ""
    req = urllib.request.Request(_url(a.controller, "/start" + q), method="POST", data=b"")
    try:
        print(urllib.request.urlopen(req, timeout=10).read().decode())
        return 0
    except urllib.error.HTTPError as e:
        print(f"refused ({e.code}): {e.read().decode(errors='replace')}", file=sys.stderr)
        return 1


def _launch(a) -> int:
    from .parallel.launcher import LocalLauncher
    cmd = a.command[1:] if a.command and a.command[0] == "--" else a.command
    if not cmd:
        print("launch: missing command after --", file=sys.stderr)
        return 2
    r = LocalLauncher(cmd, a.devices.split(","), a.policy, a.max_restarts).run()
    print(json.dumps(r.__dict__))
    return 0 if r.ok else 1


_SCAFFOLD = '''"""{name}: a flodl_b200 training script (generated by `python -m flodl_b200 init`)."""
import torch

from flodl_b200 import FlowBuilder
from flodl_b200.nn import GELU, Linear, mse_loss
from flodl_b200.optim import Adam


def main(steps: int = 200):
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    model = (FlowBuilder.from_(Linear(2, 16, device=dev)).through(GELU())
             .through(Linear(16, 2, device=dev)).build())
    opt = Adam(list(model.parameters()), lr=1e-2)
    x = torch.randn(256, 2, device=dev)
    y = torch.stack([x[:, 0] + x[:, 1], x[:, 0] - x[:, 1]], 1)
    for step in range(steps):
        loss = mse_loss(model(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        if step % 50 == 0:
            print(f"step {{step}} loss {{loss.item():.4f}}")


if __name__ == "__main__":
    main()
'''


def _init(a) -> int:
    d = a.name
    if os.path.exists(d):
        print(f"init: {d} already exists", file=sys.stderr)
        return 1
    os.makedirs(d)
    with open(os.path.join(d, "train.py"), "w") as f:
        f.write(_SCAFFOLD.format(name=os.path.basename(d)))
    print(f"created {d}/train.py - run it with `python {d}/train.py`")
    return 0


_BASH = """_flodl_b200() {
  local cur=${COMP_WORDS[COMP_CWORD]}
  if [ $COMP_CWORD -eq 1 ]; then
    COMPREPLY=( $(compgen -W "%s" -- "$cur") )
  else
    COMPREPLY=( $(compgen -W "--json --devices --policy --token --max-restarts" -- "$cur") )
  fi
}
complete -F _flodl_b200 flodl_b200
"""


def _completions(a) -> int:
    if a.shell != "bash":
        print("completions: only bash is generated", file=sys.stderr)
        return 2
    print(_BASH % " ".join(COMMANDS))
    return 0


def _commands(a) -> int:
    from .manifest import list_commands, split_env
    env, _ = split_env(a.rest)
    for k, v in list_commands(".", env).items():
        print(f"{k:16s} {v}")
    return 0


def _run(a) -> int:
    from .manifest import run, split_env
    from .schema import load_cached, validate_tail
    env, rest = split_env(a.rest)
    extra = rest[1:] if rest and rest[0] == "--" else rest
    sch = load_cached(".", a.name)
    if sch is not None:
        errs = validate_tail(sch, extra)
        if errs:
            for e in errs:
                print(f"{a.name}: {e}", file=sys.stderr)
            return 2
    return run(a.name, extra, ".", env, a.dry_run)


def _schema(a) -> int:
    from .schema import main_schema
    return main_schema(a.rest)


def _config(a) -> int:
    from .manifest import show_config, split_env
    env, rest = split_env(a.rest)
    if not rest or rest[0] in ("-h", "--help"):
        print("usage: config show [<env>|@env]")
        return 0 if rest else 1
    if rest[0] != "show":
        print(f"unknown config sub-command: {rest[0]}", file=sys.stderr)
        return 1
    env = rest[1] if len(rest) > 1 else env
    try:
        for line in show_config(".", env):
            print(line)
    except FileNotFoundError as e:
        print(f"error: {e}", file=sys.stderr)
        return 1
    return 0


def _join(a) -> int:
    from .parallel.agent import run_agent
    key = bytes.fromhex(a.key_hex or os.environ.get("FLODL_INTERNAL_KEY", ""))
    return run_agent(a.controller, key, a.devices)


def api_reference(module: str = "flodl_b200") -> dict:
    """{module: {public name: first docstring line}} for a package tree."""
    import importlib
    import inspect
    import pkgutil
    root = importlib.import_module(module)
    mods = [root]
    if hasattr(root, "__path__"):
        for info in pkgutil.walk_packages(root.__path__, module + "."):
            if info.name.split(".")[-1].startswith("_") or ".csrc" in info.name:
                continue
            try:
                mods.append(importlib.import_module(info.name))
            except Exception:
                continue
    out = {}
    for m in mods:
        names = {}
        for n, obj in vars(m).items():
            if n.startswith("_") or getattr(obj, "__module__", None) != m.__name__:
                continue
            if inspect.isclass(obj) or inspect.isfunction(obj):
                doc = inspect.cleandoc(obj.__doc__ or "").strip().splitlines()  # own docstring only
                names[n] = doc[0] if doc else ""
        if names:
            out[m.__name__] = dict(sorted(names.items()))
    return out


def _api_ref(a) -> int:
    ref = api_reference(a.module)
    if a.json:
        print(json.dumps(ref, indent=2))
    else:
        for mod, names in ref.items():
            print(f"## {mod}")
            for n, d in names.items():
                print(f"  {n}: {d}")
    return 0


_HF_PLAYGROUND = """\"\"\"HuggingFace playground: load a local model directory or a cached Hub id
and run it (generated by `python -m flodl_b200 add hf`).\"\"\"
import sys

import torch

from flodl_b200.hf import AutoModelForSequenceClassification, HfTokenizer

name = sys.argv[1] if len(sys.argv) > 1 else "distilbert-base-uncased"
model = AutoModelForSequenceClassification.from_pretrained(name).eval()
tok = HfTokenizer.from_pretrained(name)
batch = tok.encode(["flodl_b200 runs this on a B200", "and on the CPU"])
with torch.no_grad():
    print(model(batch.input_ids, attention_mask=batch.attention_mask))
"""


def _add(a) -> int:
    if a.target not in ("hf", "flodl-hf"):
        print(f"add: unknown target {a.target!r} (supported: hf)", file=sys.stderr)
        return 2
    d = os.path.join(a.dir, "flodl-hf")
    if os.path.exists(d):
        print(f"add: {d} already exists", file=sys.stderr)
        return 1
    os.makedirs(d)
    with open(os.path.join(d, "main.py"), "w") as f:
        f.write(_HF_PLAYGROUND)
    with open(os.path.join(d, "fdl.yml"), "w") as f:
        f.write("commands:\n  run:\n    description: run the HF playground\n    run: python main.py\n")
    manifest = os.path.join(a.dir, "fdl.yml")
    entry = "  flodl-hf:                     # sub-manifest ./flodl-hf/fdl.yml\n"
    if os.path.exists(manifest):
        text = open(manifest).read()
        if "flodl-hf:" not in text:
            if "commands:" not in text:
                text += "\ncommands:\n"
            text = text.replace("commands:\n", "commands:\n" + entry, 1)
            open(manifest, "w").write(text)
    else:
        open(manifest, "w").write("commands:\n" + entry)
    print(f"created {d}/ (run it with `python -m flodl_b200 run flodl-hf:run`)")
    return 0


def publish(src: str, dest: str) -> dict:
    """Validate a run directory (its Python files compile, its fdl.yml parses)
    and publish it into ``dest`` with a ``run.json`` manifest agents read."""
    import hashlib
    import py_compile
    import shutil
    import time
    files = []
    for root, _, fs in os.walk(src):
        for f in fs:
            p = os.path.join(root, f)
            if f.endswith(".py"):
                py_compile.compile(p, doraise=True)
            files.append(os.path.relpath(p, src))
    if os.path.exists(os.path.join(src, "fdl.yml")):
        from .manifest import load_manifest
        load_manifest(src)
    h = hashlib.sha256()
    for f in sorted(files):
        h.update(f.encode())
        h.update(open(os.path.join(src, f), "rb").read())
    digest = h.hexdigest()[:16]
    target = os.path.join(dest, f"run-{digest}")
    if not os.path.exists(target):
        shutil.copytree(src, target + ".tmp")
        os.replace(target + ".tmp", target)
    man = {"run": os.path.basename(target), "digest": digest, "files": sorted(files),
           "published_at": time.time()}
    tmp = os.path.join(dest, "run.json.tmp")
    with open(tmp, "w") as f:
        json.dump(man, f, indent=2)
    os.replace(tmp, os.path.join(dest, "run.json"))
    return man


def _publish(a) -> int:
    try:
        man = publish(a.src, a.dest)
    except Exception as e:
        print(f"publish: refused: {e}", file=sys.stderr)
        return 1
    print(json.dumps(man))
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m flodl_b200",
                                 description="flodl_b200 command line")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("probe", help="hardware survey")
    p.add_argument("--json", action="store_true")
    p = sub.add_parser("diagnose", help="environment checks")
    p.add_argument("--json", action="store_true")
    p = sub.add_parser("status", help="controller state.json")
    p.add_argument("controller")
    p.add_argument("--json", action="store_true")
    p = sub.add_parser("start", help="arm a manual start")
    p.add_argument("controller")
    p.add_argument("--token", default="")
    p = sub.add_parser("launch", help="one process per device")
    p.add_argument("--devices", required=True)
    p.add_argument("--policy", default="abort", choices=["abort", "shrink"])
    p.add_argument("--max-restarts", type=int, default=1)
    p.add_argument("command", nargs=argparse.REMAINDER)
    p = sub.add_parser("init", help="scaffold a training script")
    p.add_argument("name")
    p = sub.add_parser("completions", help="shell completion script")
    p.add_argument("shell")
    p = sub.add_parser("commands", help="list fdl.yml commands")
    p.add_argument("rest", nargs=argparse.REMAINDER)
    p = sub.add_parser("run", help="run an fdl.yml command")
    p.add_argument("name")
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("rest", nargs=argparse.REMAINDER)
    p = sub.add_parser("join", help="join a controller as this host's agent")
    p.add_argument("controller")
    p.add_argument("--key-hex", default="")
    p.add_argument("--devices", type=int, default=None)
    p = sub.add_parser("api-ref", help="public API surface")
    p.add_argument("module", nargs="?", default="flodl_b200")
    p.add_argument("--json", action="store_true")
    p = sub.add_parser("add", help="scaffold an add-on playground")
    p.add_argument("target")
    p.add_argument("--dir", default=".")
    p = sub.add_parser("publish", help="validate and publish a run directory")
    p.add_argument("src")
    p.add_argument("dest")
    p = sub.add_parser("schema", help="cached --fdl-schema outputs: list | clear | refresh")
    p.add_argument("rest", nargs=argparse.REMAINDER)
    p = sub.add_parser("config", help="config show [<env>]: the merged fdl.yml with sources")
    p.add_argument("rest", nargs=argparse.REMAINDER)
    return ap


def main(argv=None) -> int:
    a = build_parser().parse_args(argv)
    return {"probe": _probe, "diagnose": _diagnose, "status": _status, "start": _start,
            "launch": _launch, "init": _init, "completions": _completions,
            "commands": _commands, "run": _run, "join": _join, "api-ref": _api_ref, "add": _add,
            "publish": _publish, "schema": _schema, "config": _config}[a.cmd](a)
