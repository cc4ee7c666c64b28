"""Declarative command-line arguments with a machine-readable schema.

The reference's ``#[derive(FdlArgs)]`` (flodl-cli-macros/src/lib.rs, parser
in flodl-cli/src/args/) turns one struct into an argv parser, a help text and
a JSON schema that the ``fdl`` driver caches and validates against. Here the
struct is a dataclass whose fields carry :func:`option` / :func:`arg`
metadata::

    @dataclass
    class TrainArgs:
        \"\"\"Train a model.\"\"\"
        model: str = option("mlp", short="m", choices=["mlp", "resnet"],
                            help="Model architecture to use.")
        epochs: int = option(10, short="e", help="Number of epochs.")
        wandb_key: Optional[str] = option(None, env="WANDB_API_KEY", help="API key.")
        datasets: List[str] = arg(variadic=True, help="Extra dataset paths.")

    args = parse_or_schema(TrainArgs)

``--fdl-schema`` anywhere in argv prints the schema and exits 0; ``--help``
prints the help. Field types give the cardinality the reference uses:
``bool`` flags (absent = False), scalars, ``Optional[T]`` (absent = None),
``List[T]`` (repeatable option / variadic last positional). Option names are
the kebab-cased field names. The schema keeps the reference's JSON shape
(``{"args": [...], "options": {name: {...}}}``, types ``string``, ``int``,
``float``, ``bool``, ``path``, ``list[...]``) so the driver's caches and
validation (``schema.py``) read either.
"""
from __future__ import annotations

import dataclasses
import json
import os
import pathlib
import sys
import typing
from typing import Any, Dict, List, Optional, Sequence, Type, TypeVar

T = TypeVar("T")

RESERVED_LONGS = ("help", "version", "quiet", "env", "fdl-schema")
RESERVED_SHORTS = ("h", "V", "q")
_MISSING = dataclasses.MISSING


class ArgsError(ValueError):
    """A command line that does not match the declared arguments."""


def option(default: Any = _MISSING, *, short: Optional[str] = None,
           choices: Optional[Sequence[Any]] = None, env: Optional[str] = None,
           help: str = "", completer: Optional[str] = None):
    """A named ``--kebab-name`` option (bool fields are flags)."""
    meta = {"fdl": "option", "short": short, "choices": list(choices) if choices else None,
            "env": env, "help": help, "completer": completer}
    if default is _MISSING:
        return dataclasses.field(metadata=meta)
    if isinstance(default, list):
        return dataclasses.field(default_factory=lambda d=default: list(d), metadata=meta)
    return dataclasses.field(default=default, metadata=meta)


def arg(default: Any = _MISSING, *, variadic: bool = False,
        choices: Optional[Sequence[Any]] = None, help: str = "",
        completer: Optional[str] = None):
    """A positional argument (``variadic``: the last one, collecting the rest)."""
    meta = {"fdl": "arg", "variadic": variadic, "choices": list(choices) if choices else None,
            "help": help, "completer": completer}
    if variadic and default is _MISSING:
        return dataclasses.field(default_factory=list, metadata=meta)
    if default is _MISSING:
        return dataclasses.field(metadata=meta)
    return dataclasses.field(default=default, metadata=meta)


# ------------------------------------------------------------------ types
def _unwrap(tp) -> tuple:
    """(base type, optional, is_list) of a field annotation."""
    origin = typing.get_origin(tp)
    if origin is typing.Union:
        inner = [a for a in typing.get_args(tp) if a is not type(None)]
        base, _, is_list = _unwrap(inner[0])
        return base, True, is_list
    if origin in (list, List):
        (inner,) = typing.get_args(tp) or (str,)
        return inner, False, True
    return tp, False, False


def _type_name(base) -> str:
    if base is bool:
        return "bool"
    if base is int:
        return "int"
    if base is float:
        return "float"
    if base in (pathlib.Path, os.PathLike):
        return "path"
    return "string"


def _convert(base, text: str, where: str):
    try:
        if base is bool:
            low = text.lower()
            if low in ("1", "true", "yes", "on"):
                return True
            if low in ("0", "false", "no", "off"):
                return False
            raise ValueError(text)
        if base is int:
            return int(text)
        if base is float:
            return float(text)
        if base is pathlib.Path:
            return pathlib.Path(text)
        return text
    except ValueError:
        raise ArgsError(f"{where}: invalid {_type_name(base)} value {text!r}") from None


def _kebab(name: str) -> str:
    return name.replace("_", "-")


class _Spec:
    def __init__(self, cls):
        if not dataclasses.is_dataclass(cls):
            raise TypeError(f"{cls.__name__} must be a dataclass")
        hints = typing.get_type_hints(cls)
        self.cls = cls
        self.options: Dict[str, dict] = {}
        self.args: List[dict] = []
        shorts: Dict[str, str] = {}
        for f in dataclasses.fields(cls):
            meta = dict(f.metadata) if f.metadata else {"fdl": "option", "help": ""}
            base, optional, is_list = _unwrap(hints[f.name])
            has_default = f.default is not _MISSING or f.default_factory is not _MISSING
            default = (f.default if f.default is not _MISSING else
                       f.default_factory() if f.default_factory is not _MISSING else None)
            ty = _type_name(base)
            if is_list:
                ty = f"list[{ty}]"
            rec = dict(field=f.name, base=base, optional=optional, is_list=is_list, type=ty,
                       default=default, has_default=has_default, **meta)
            if meta["fdl"] == "option":
                name = _kebab(f.name)
                if name in RESERVED_LONGS:
                    raise TypeError(f"option --{name} is reserved")
                s = meta.get("short")
                if s:
                    if len(s) != 1 or s in RESERVED_SHORTS:
                        raise TypeError(f"short -{s} of --{name} is invalid or reserved")
                    if s in shorts:
                        raise TypeError(f"short -{s} used by --{shorts[s]} and --{name}")
                    shorts[s] = name
                if not has_default and not optional and base is not bool and not is_list:
                    raise TypeError(f"option --{name} needs a default (or Optional[...])")
                self.options[name] = rec
            else:
                if self.args and self.args[-1].get("variadic"):
                    raise TypeError("a variadic positional must be the last one")
                self.args.append(rec)
        self.shorts = shorts

    # ---------------------------------------------------------------- schema
    def schema(self) -> dict:
        out: Dict[str, Any] = {}
        if self.args:
            args = []
            for a in self.args:
                d = {"name": a["field"], "type": a["type"]}
                if a.get("help"):
                    d["description"] = a["help"]
                d["required"] = not (a["has_default"] or a["optional"] or a["variadic"])
                if a["variadic"]:
                    d["variadic"] = True
                if a["has_default"] and not a["variadic"] and a["default"] is not None:
                    d["default"] = _jsonable(a["default"])
                if a.get("choices"):
                    d["choices"] = [_jsonable(c) for c in a["choices"]]
                if a.get("completer"):
                    d["completer"] = a["completer"]
                args.append(d)
            out["args"] = args
        if self.options:
            opts = {}
            for name in sorted(self.options):
                o = self.options[name]
                d = {"type": o["type"]}
                if o.get("help"):
                    d["description"] = o["help"]
                if o["has_default"] and o["default"] is not None and o["default"] != []:
                    d["default"] = _jsonable(o["default"])
                for k in ("choices", "short", "env", "completer"):
                    if o.get(k):
                        d[k] = [_jsonable(c) for c in o[k]] if k == "choices" else o[k]
                opts[name] = d
            out["options"] = opts
        return out

    # ---------------------------------------------------------------- help
    def help(self, prog: str) -> str:
        doc = (self.cls.__doc__ or "").strip()
        if doc.startswith(self.cls.__name__ + "("):  # dataclass auto-doc
            doc = ""
        usage = [prog]
        if self.options:
            usage.append("[OPTIONS]")
        for a in self.args:
            n = a["field"].upper()
            usage.append(f"[{n}...]" if a["variadic"] else (f"[{n}]" if not
                                                             _required(a) else f"<{n}>"))
        lines = []
        if doc:
            lines += [doc, ""]
        lines.append("Usage: " + " ".join(usage))
        if self.args:
            lines += ["", "Arguments:"]
            for a in self.args:
                lines.append(f"  {a['field']:<22} {a.get('help', '')}")
        lines += ["", "Options:"]
        for name in sorted(self.options):
            o = self.options[name]
            flag = (f"-{o['short']}, " if o.get("short") else "    ") + f"--{name}"
            if o["base"] is not bool or o["is_list"]:
                flag += f" <{o['type']}>"
            extra = []
            if o["has_default"] and o["default"] not in (None, [], False):
                extra.append(f"default: {o['default']}")
            if o.get("choices"):
                extra.append("choices: " + ", ".join(map(str, o["choices"])))
            if o.get("env"):
                extra.append(f"env: {o['env']}")
            tail = f" [{'; '.join(extra)}]" if extra else ""
            lines.append(f"  {flag:<28} {o.get('help', '')}{tail}")
        lines.append(f"  {'-h, --help':<28} Print help")
        lines.append(f"  {'--fdl-schema':<28} Print the argument schema (JSON)")
        return "\n".join(lines)

    # ---------------------------------------------------------------- parse
    def parse(self, argv: Sequence[str]):
        values: Dict[str, Any] = {}
        positional: List[str] = []
        i = 0
        argv = list(argv)
        only_pos = False
        while i < len(argv):
            tok = argv[i]
            i += 1
            if only_pos or not tok.startswith("-") or tok == "-":
                positional.append(tok)
                continue
            if tok == "--":
                only_pos = True
                continue
            if tok.startswith("--"):
                name, eq, inline = tok[2:].partition("=")
                if name not in self.options:
                    raise ArgsError(f"unknown option --{name}" + _suggest(name, self.options))
            else:
                s = tok[1:2]
                if s not in self.shorts:
                    raise ArgsError(f"unknown option -{s}")
                name = self.shorts[s]
                eq, inline = ("=", tok[2:]) if len(tok) > 2 else ("", "")
            o = self.options[name]
            if o["base"] is bool and not o["is_list"]:
                values[o["field"]] = _convert(bool, inline, f"--{name}") if eq else True
                continue
            if eq:
                text = inline
            else:
                if i >= len(argv):
                    raise ArgsError(f"--{name} needs a value")
                text = argv[i]
                i += 1
            v = _convert(o["base"], text, f"--{name}")
            _check_choice(o, v, f"--{name}")
            if o["is_list"]:
                values.setdefault(o["field"], []).append(v)
            else:
                values[o["field"]] = v
        # environment fallbacks, then defaults
        for name, o in self.options.items():
            f = o["field"]
            if f in values:
                continue
            if o.get("env") and os.environ.get(o["env"]) is not None:
                raw = os.environ[o["env"]]
                if o["is_list"]:
                    values[f] = [_convert(o["base"], x, o["env"]) for x in raw.split(",") if x]
                else:
                    values[f] = _convert(o["base"], raw, o["env"])
                    _check_choice(o, values[f], o["env"])
            elif o["base"] is bool and not o["is_list"] and not o["has_default"]:
                values[f] = False
            elif not o["has_default"]:
                values[f] = [] if o["is_list"] else None
        # positionals
        for a in self.args:
            f = a["field"]
            if a["variadic"]:
                vals = [_convert(a["base"], t, a["field"]) for t in positional]
                for v in vals:
                    _check_choice(a, v, a["field"])
                values[f] = vals
                positional = []
                continue
            if positional:
                v = _convert(a["base"], positional.pop(0), a["field"])
                _check_choice(a, v, a["field"])
                values[f] = v
            elif _required(a):
                raise ArgsError(f"missing required argument <{a['field']}>")
        if positional:
            raise ArgsError(f"unexpected argument {positional[0]!r}")
        return self.cls(**values)


def _required(a) -> bool:
    return not (a["has_default"] or a["optional"] or a["variadic"])


def _check_choice(rec, v, where):
    ch = rec.get("choices")
    if ch and v not in ch:
        raise ArgsError(f"{where}: {v!r} is not one of {', '.join(map(str, ch))}")


def _suggest(name: str, known) -> str:
    import difflib
    m = difflib.get_close_matches(name, list(known), n=1)
    return f" (did you mean --{m[0]}?)" if m else ""


def _jsonable(v):
    return str(v) if isinstance(v, pathlib.Path) else v


# ------------------------------------------------------------------ entry points
def schema_of(cls: Type[T]) -> dict:
    """The JSON schema of a declared argument dataclass."""
    return _Spec(cls).schema()


def help_of(cls: Type[T], prog: str = "prog") -> str:
    return _Spec(cls).help(prog)


def try_parse(cls: Type[T], argv: Sequence[str]) -> T:
    """Parse ``argv`` (without the program name); raises :class:`ArgsError`."""
    return _Spec(cls).parse(argv)


def parse_or_schema(cls: Type[T], argv: Optional[Sequence[str]] = None) -> T:
    """``--fdl-schema``: print the schema and exit 0; ``--help``/``-h``: print
    the help and exit 0; otherwise parse, and on an error print the message
    and the help to stderr and exit 2 (the reference's ``parse_or_schema``)."""
    argv = list(sys.argv if argv is None else argv)
    prog, rest = (os.path.basename(argv[0]) if argv else "prog"), argv[1:]
    spec = _Spec(cls)
    before = rest[:rest.index("--")] if "--" in rest else rest
    if "--fdl-schema" in before:
        print(json.dumps(spec.schema(), indent=2))
        raise SystemExit(0)
    if "--help" in before or "-h" in before:
        print(spec.help(prog))
        raise SystemExit(0)
    try:
        return spec.parse(rest)
    except ArgsError as e:
        print(str(e), file=sys.stderr)
        print("", file=sys.stderr)
        print(spec.help(prog), file=sys.stderr)
        raise SystemExit(2)
