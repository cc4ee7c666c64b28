"""``--fdl-schema`` contract: probe a command, validate its schema, cache it.

Role of flodl-cli/src/schema_cache.rs and the ``fdl schema`` subcommand
(flodl-cli/src/cli/schema.rs): a command of ``fdl.yml`` whose program was
written with :mod:`flodl_b200.args` answers ``--fdl-schema`` with its argument
schema. The driver caches that JSON under ``<project>/.fdl/schema-cache/
<cmd>.json``; a cache older than ``fdl.yml`` (or any overlay) or than the
script the command runs is *stale*, a cache whose command left the manifest
is an *orphan*. :func:`validate_tail` checks a command line against a schema
(unknown options with a suggestion, values outside ``choices``) before the
command runs.
"""
from __future__ import annotations

import difflib
import glob
import json
import os
import shlex
import subprocess
import sys
from dataclasses import dataclass
from typing import List, Optional

from . import manifest

CACHE_DIR = os.path.join(".fdl", "schema-cache")


@dataclass
class CacheEntry:
    cmd_name: str
    cache_path: str
    status: str  # fresh | stale | orphan


def cache_path(project: str, cmd: str) -> str:
    return os.path.join(project, CACHE_DIR, cmd.replace(":", "__") + ".json")


def check_schema(obj) -> dict:
    """Shape check: ``{"args": [...], "options": {...}}``, both optional."""
    if not isinstance(obj, dict):
        raise ValueError("schema must be a JSON object")
    args = obj.get("args", [])
    opts = obj.get("options", {})
    if not isinstance(args, list) or not isinstance(opts, dict):
        raise ValueError("schema needs a list 'args' and a mapping 'options'")
    for a in args:
        if not isinstance(a, dict) or "name" not in a or "type" not in a:
            raise ValueError(f"bad positional spec {a!r}")
    for k, o in opts.items():
        if not isinstance(o, dict) or "type" not in o:
            raise ValueError(f"bad option spec for {k!r}")
    return obj


def source_refs(project: str, cmd: str) -> List[str]:
    """Files whose change may change the command's schema: the manifests and
    every existing file named on the command's ``run`` line."""
    refs = sorted(glob.glob(os.path.join(project, "fdl*.yml")))
    try:
        spec, d = manifest.resolve(manifest.load_manifest(project), cmd, project)
    except (KeyError, FileNotFoundError):
        return refs
    for tok in shlex.split(spec.get("run", "")):
        p = os.path.join(d, spec.get("cwd", "."), tok)
        if os.path.isfile(p):
            refs.append(p)
        elif tok.count(".") and not tok.startswith("-"):
            # `python -m pkg.mod`: the module file, when it is in the project
            cand = os.path.join(project, *tok.split(".")) + ".py"
            if os.path.isfile(cand):
                refs.append(cand)
    return refs


def status(project: str, cmd: str, known: Optional[set] = None) -> str:
    path = cache_path(project, cmd)
    if known is not None and cmd not in known:
        return "orphan"
    mtime = os.path.getmtime(path)
    for r in source_refs(project, cmd):
        if os.path.getmtime(r) > mtime:
            return "stale"
    return "fresh"


def discover(project: str = ".") -> List[CacheEntry]:
    d = os.path.join(project, CACHE_DIR)
    if not os.path.isdir(d):
        return []
    try:
        known = set(manifest.list_commands(project))
    except FileNotFoundError:
        known = set()
    out = []
    for f in sorted(os.listdir(d)):
        if f.endswith(".json"):
            cmd = f[:-5].replace("__", ":")
            out.append(CacheEntry(cmd, os.path.join(d, f), status(project, cmd, known)))
    return out


def probe(project: str, cmd: str, timeout: float = 60.0) -> dict:
    """Run ``<command> --fdl-schema`` and return the validated schema."""
    m = manifest.load_manifest(project)
    spec, d = manifest.resolve(m, cmd, project)
    line = manifest.command_line(spec, ["--fdl-schema"])
    env = dict(os.environ)
    env.update({k: str(v) for k, v in (m.get("env") or {}).items()})
    env.update({k: str(v) for k, v in (spec.get("env") or {}).items()})
    r = subprocess.run(line, shell=True, cwd=os.path.join(d, spec.get("cwd", ".")), env=env,
                       capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"{cmd}: --fdl-schema exited {r.returncode}: {r.stderr.strip()[-300:]}")
    try:
        return check_schema(json.loads(r.stdout))
    except json.JSONDecodeError as e:
        raise RuntimeError(f"{cmd}: --fdl-schema printed no JSON ({e})") from None


def refresh(project: str = ".", cmd: Optional[str] = None) -> List[str]:
    """Probe and cache one command, or every command that answers. Returns
    the commands cached."""
    names = [cmd] if cmd else [n for n, v in manifest.load_manifest(project)["commands"].items()
                               if v is not None]
    done = []
    for n in names:
        try:
            sch = probe(project, n)
        except (RuntimeError, subprocess.TimeoutExpired, KeyError) as e:
            if cmd:
                raise RuntimeError(str(e)) from None
            continue
        path = cache_path(project, n)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        tmp = path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(sch, f, indent=2, sort_keys=True)
        os.replace(tmp, path)
        done.append(n)
    return done


def clear(project: str = ".", cmd: Optional[str] = None) -> int:
    n = 0
    for e in discover(project):
        if cmd is None or e.cmd_name == cmd:
            os.remove(e.cache_path)
            n += 1
    return n


def load_cached(project: str, cmd: str) -> Optional[dict]:
    p = cache_path(project, cmd)
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return check_schema(json.load(f))


def validate_tail(schema: dict, tail: List[str]) -> List[str]:
    """Problems of a command line against a schema (empty: fine). Unknown
    long options get a did-you-mean; declared ``choices`` are enforced."""
    opts = schema.get("options", {})
    shorts = {o["short"]: k for k, o in opts.items() if o.get("short")}
    errs = []
    i = 0
    while i < len(tail):
        tok = tail[i]
        i += 1
        if tok == "--":
            break
        if tok.startswith("--"):
            name, eq, val = tok[2:].partition("=")
            if name in ("help", "fdl-schema"):
                continue
            if name not in opts:
                m = difflib.get_close_matches(name, list(opts), n=1)
                errs.append(f"unknown option --{name}" + (f" (did you mean --{m[0]}?)" if m else ""))
                continue
        elif tok.startswith("-") and len(tok) > 1 and tok != "-":
            s = tok[1]
            if s == "h":
                continue
            if s not in shorts:
                errs.append(f"unknown option -{s}")
                continue
            name = shorts[s]
            eq, val = ("=", tok[2:]) if len(tok) > 2 else ("", "")
        else:
            continue
        o = opts[name]
        if o["type"] == "bool":
            continue
        if not eq:
            if i >= len(tail):
                errs.append(f"--{name} needs a value")
                break
            val = tail[i]
            i += 1
        ch = o.get("choices")
        if ch and val not in [str(c) for c in ch]:
            errs.append(f"--{name}: {val!r} is not one of {', '.join(map(str, ch))}")
    return errs


def main_schema(argv: List[str], project: str = ".") -> int:
    """``schema list [--json] | clear [cmd] | refresh [cmd]``."""
    sub = argv[0] if argv else "--help"
    if sub == "list":
        entries = discover(project)
        if "--json" in argv:
            print(json.dumps([{"name": e.cmd_name, "path": os.path.relpath(e.cache_path, project),
                               "status": e.status} for e in entries]))
        elif not entries:
            print(f"No cached schemas under {os.path.abspath(project)}.")
            print("Run `python -m flodl_b200 schema refresh` to populate.")
        else:
            for e in entries:
                print(f"{e.cmd_name:<24} {e.status:<7} {os.path.relpath(e.cache_path, project)}")
        return 0
    if sub == "clear":
        n = clear(project, argv[1] if len(argv) > 1 else None)
        print(f"cleared {n} cached schema(s)")
        return 0
    if sub == "refresh":
        try:
            done = refresh(project, argv[1] if len(argv) > 1 else None)
        except RuntimeError as e:
            print(f"error: {e}", file=sys.stderr)
            return 1
        print(f"cached {len(done)} schema(s): {', '.join(done) if done else '-'}")
        return 0
    print("usage: schema list [--json] | schema clear [<cmd>] | schema refresh [<cmd>]")
    return 0 if sub in ("--help", "-h") else 1
