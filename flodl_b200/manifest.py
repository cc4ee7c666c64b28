"""Command manifests: ``fdl.yml`` with environment overlays.

Reference role: flodl-cli's manifest and overlay system
(flodl-cli/src/config/*.rs, overlay.rs, fdl.yml.example): a project's
commands live in ``fdl.yml`` under ``commands: {name: {description, run,
append, env, cwd}}``; ``fdl.<env>.yml`` overlays are deep-merged on top when
an environment is selected (``@env`` on the command line, or ``FDL_ENV``); a
command whose body is empty delegates to the child manifest
``./<name>/fdl.yml``. Mappings merge key by key, anything else in the overlay
replaces the base value, and a ``null`` in the overlay deletes the key.
"""
from __future__ import annotations

import json
import os
import shlex
import subprocess
from typing import Dict, List, Optional, Tuple

import yaml

ENV_VAR = "FDL_ENV"


def deep_merge(base, over):
    if isinstance(base, dict) and isinstance(over, dict):
        out = dict(base)
        for k, v in over.items():
            if v is None:
                out.pop(k, None)
            elif k in out:
                out[k] = deep_merge(out[k], v)
            else:
                out[k] = v
        return out
    return over


def load_manifest(directory: str = ".", env: Optional[str] = None) -> dict:
    path = os.path.join(directory, "fdl.yml")
    with open(path) as f:
        m = yaml.safe_load(f) or {}
    env = env or os.environ.get(ENV_VAR)
    if env:
        op = os.path.join(directory, f"fdl.{env}.yml")
        if not os.path.exists(op):
            raise FileNotFoundError(f"overlay fdl.{env}.yml not found in {directory}")
        with open(op) as f:
            m = deep_merge(m, yaml.safe_load(f) or {})
    m.setdefault("commands", {})
    return m


def config_layers(directory: str = ".", env: Optional[str] = None) -> List[Tuple[str, dict]]:
    """The files that make up the resolved manifest, base first: ``fdl.yml``,
    then the ``fdl.<env>.yml`` overlay when an environment is selected."""
    layers = []
    with open(os.path.join(directory, "fdl.yml")) as f:
        layers.append(("fdl.yml", yaml.safe_load(f) or {}))
    env = env or os.environ.get(ENV_VAR)
    if env:
        op = os.path.join(directory, f"fdl.{env}.yml")
        if not os.path.exists(op):
            raise FileNotFoundError(f"overlay fdl.{env}.yml not found in {directory}")
        with open(op) as f:
            layers.append((f"fdl.{env}.yml", yaml.safe_load(f) or {}))
    return layers


def show_config(directory: str = ".", env: Optional[str] = None) -> List[str]:
    """The merged manifest, one leaf per line (``dotted.key: value``), each
    tagged with the file that set it (the reference's ``fdl config show``)."""
    layers = config_layers(directory, env)
    merged, source = {}, {}

    def walk(node, prefix, label):
        for k, v in (node or {}).items():
            key = f"{prefix}.{k}" if prefix else str(k)
            if v is None:  # an overlay null deletes the key
                for s in [s for s in source if s == key or s.startswith(key + ".")]:
                    source.pop(s)
            elif isinstance(v, dict):
                walk(v, key, label)
            else:
                source[key] = label

    for label, data in layers:
        merged = deep_merge(merged, data)
        walk(data, "", label)

    def value(key):
        node = merged
        for part in key.split("."):
            node = node[part]
        return node

    width = max((len(k) for k in source), default=0)
    return [f"{k:<{width}}  {json.dumps(value(k))}  # {source[k]}" for k in sorted(source)]


def split_env(args: List[str]) -> Tuple[Optional[str], List[str]]:
    """``@env`` anywhere among the arguments selects the overlay."""
    env, rest = None, []
    for a in args:
        if a.startswith("@") and len(a) > 1 and env is None:
            env = a[1:]
        else:
            rest.append(a)
    return env, rest


def resolve(manifest: dict, name: str, directory: str = ".", env: Optional[str] = None):
    """(command spec, directory it runs in); follows child manifests for
    ``parent child`` style names given as ``parent:child``."""
    head, _, tail = name.partition(":")
    cmds = manifest.get("commands", {})
    if head not in cmds:
        raise KeyError(f"no command {head!r} (have: {', '.join(sorted(cmds))})")
    spec = cmds[head]
    if spec is None:
        child_dir = os.path.join(directory, head)
        child = load_manifest(child_dir, env)
        if not tail:
            raise KeyError(f"{head!r} is a sub-manifest; name one of its commands as {head}:<cmd>")
        return resolve(child, tail, child_dir, env)
    if isinstance(spec, str):
        spec = {"run": spec}
    return spec, directory


def command_line(spec: dict, extra: List[str]) -> str:
    cmd = spec["run"]
    if spec.get("append"):
        cmd += " " + spec["append"]
    if extra:
        cmd += " " + " ".join(shlex.quote(a) for a in extra)
    return cmd


def run(name: str, extra: List[str], directory: str = ".", env: Optional[str] = None,
        dry: bool = False) -> int:
    m = load_manifest(directory, env)
    spec, d = resolve(m, name, directory, env)
    cmd = command_line(spec, extra)
    if dry:
        print(cmd)
        return 0
    penv = dict(os.environ)
    penv.update({k: str(v) for k, v in (m.get("env") or {}).items()})
    penv.update({k: str(v) for k, v in (spec.get("env") or {}).items()})
    if env:
        penv[ENV_VAR] = env
    return subprocess.call(cmd, shell=True, cwd=os.path.join(d, spec.get("cwd", ".")), env=penv)


def list_commands(directory: str = ".", env: Optional[str] = None) -> Dict[str, str]:
    m = load_manifest(directory, env)
    out = {}
    for k, v in m["commands"].items():
        if v is None:
            out[k] = f"(sub-manifest ./{k}/fdl.yml)"
        elif isinstance(v, str):
            out[k] = v
        else:
            out[k] = v.get("description", v.get("run", ""))
    return out
