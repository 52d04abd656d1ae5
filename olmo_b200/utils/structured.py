"""
A small typed-configuration engine: YAML + dotted overrides -> validated dataclass instances.

The reference builds its configuration objects with OmegaConf structured configs
(``olmo/config.py:127-148``).  This module provides the same observable behaviour without that
dependency:

* a dataclass acts as the schema; unknown keys are rejected;
* values are coerced to the annotated type (``Enum`` by value *or* name, ``Optional``, ``Union``,
  ``Tuple``, ``List``, ``Dict``, nested dataclasses, ``"1e-6"`` -> ``float``);
* ``${a.b.c}`` interpolations are resolved against the root document, ``${oc.env:VAR[,default]}``
  against the environment, and ``${name:arg1,arg2}`` against a resolver registry
  (``path.glob``, ``path.choose`` and ``path.last_checkpoint`` are registered by
  :mod:`olmo_b200.config`);
* overrides are ``key.sub=value`` strings whose value part is parsed as YAML.

Everything here is plain Python and is exercised by the CPU test-suite.
"""
from __future__ import annotations

import dataclasses
import os
import re
import typing
from enum import Enum
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple, Type, Union

import yaml

from ..exceptions import OLMoConfigurationError

__all__ = [
    "MISSING",
    "load_yaml",
    "dump_yaml",
    "parse_dotlist",
    "deep_merge",
    "resolve_interpolations",
    "build",
    "to_container",
    "register_resolver",
]


class _Missing:
    def __repr__(self) -> str:  # pragma: no cover
        return "MISSING"


MISSING = _Missing()

# ---------------------------------------------------------------------------------------------
# YAML reading/writing.  PyYAML follows YAML 1.1 where "1e-6" is a string; training configs
# routinely write learning rates that way, so floats get a wider implicit resolver.
# ---------------------------------------------------------------------------------------------


class _Loader(yaml.SafeLoader):
    pass


_Loader.add_implicit_resolver(
    "tag:yaml.org,2002:float",
    re.compile(
        r"""^(?:
         [-+]?(?:[0-9][0-9_]*)\.[0-9_]*(?:[eE][-+]?[0-9]+)?
        |[-+]?(?:[0-9][0-9_]*)(?:[eE][-+]?[0-9]+)
        |\.[0-9_]+(?:[eE][-+][0-9]+)?
        |[-+]?\.(?:inf|Inf|INF)
        |\.(?:nan|NaN|NAN))$""",
        re.X,
    ),
    list("-+0123456789."),
)


def load_yaml(text_or_stream: Any) -> Any:
    """Parse YAML with scientific-notation floats recognised."""
    return yaml.load(text_or_stream, Loader=_Loader)


class _Dumper(yaml.SafeDumper):
    pass


def _represent_enum(dumper: yaml.Dumper, data: Enum):
    # OmegaConf writes the member *name*; for string enums name == value in every config class.
    return dumper.represent_str(data.name)


_Dumper.add_multi_representer(Enum, _represent_enum)
_Dumper.add_representer(tuple, lambda d, v: d.represent_list(list(v)))


def dump_yaml(obj: Any) -> str:
    return yaml.dump(obj, Dumper=_Dumper, default_flow_style=False, sort_keys=False, allow_unicode=True)


# ---------------------------------------------------------------------------------------------
# Dotted overrides and merging.
# ---------------------------------------------------------------------------------------------


def parse_dotlist(items: Sequence[str]) -> Dict[str, Any]:
    """``["a.b=1", "c=[1,2]"]`` -> ``{"a": {"b": 1}, "c": [1, 2]}``."""
    out: Dict[str, Any] = {}
    for item in items:
        if "=" not in item:
            key, raw = item, None
        else:
            key, raw = item.split("=", 1)
        key = key.strip()
        if not key:
            raise OLMoConfigurationError(f"bad override '{item}'")
        if raw is None or raw == "":
            value: Any = None
        elif "${" in raw:
            value = raw  # keep interpolations verbatim
        else:
            try:
                value = load_yaml(raw)
            except yaml.YAMLError:
                value = raw
        node = out
        parts = key.split(".")
        for p in parts[:-1]:
            nxt = node.get(p)
            if not isinstance(nxt, dict):
                nxt = {}
                node[p] = nxt
            node = nxt
        node[parts[-1]] = value
    return out


def deep_merge(base: Any, update: Any) -> Any:
    """Recursive dict merge; lists and scalars in ``update`` replace those in ``base``.

    A numeric-string key into a list (``evaluators.0.label=x``) updates that list element.
    """
    if isinstance(base, dict) and isinstance(update, dict):
        merged = dict(base)
        for k, v in update.items():
            merged[k] = deep_merge(merged[k], v) if k in merged else v
        return merged
    if isinstance(base, list) and isinstance(update, dict) and all(str(k).isdigit() for k in update):
        merged_list = list(base)
        for k, v in update.items():
            i = int(k)
            if i >= len(merged_list):
                raise OLMoConfigurationError(f"override index {i} out of range")
            merged_list[i] = deep_merge(merged_list[i], v)
        return merged_list
    return update


# ---------------------------------------------------------------------------------------------
# Interpolation.
# ---------------------------------------------------------------------------------------------

_RESOLVERS: Dict[str, Callable[..., Any]] = {}


def register_resolver(name: str, fn: Callable[..., Any]) -> None:
    _RESOLVERS[name] = fn


def _env_resolver(name: str, default: Any = MISSING) -> Any:
    if name in os.environ:
        return os.environ[name]
    if default is MISSING:
        raise OLMoConfigurationError(f"environment variable '{name}' is not set")
    return None if default == "null" else default


register_resolver("oc.env", _env_resolver)

_INTERP = re.compile(r"\$\{([^${}]+)\}")


def _lookup(root: Any, dotted: str) -> Any:
    node = root
    for part in dotted.split("."):
        if isinstance(node, dict):
            if part not in node:
                raise OLMoConfigurationError(f"interpolation key '{dotted}' not found")
            node = node[part]
        elif isinstance(node, list):
            node = node[int(part)]
        else:
            raise OLMoConfigurationError(f"interpolation key '{dotted}' not found")
    return node


def _split_args(s: str) -> List[str]:
    args, depth, cur = [], 0, ""
    for ch in s:
        if ch in "[{(":
            depth += 1
        elif ch in "]})":
            depth -= 1
        if ch == "," and depth == 0:
            args.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip() or args:
        args.append(cur.strip())
    return args


def _resolve_string(value: str, root: Any, depth: int = 0) -> Any:
    if depth > 32:
        raise OLMoConfigurationError(f"interpolation cycle while resolving '{value}'")

    def eval_expr(expr: str) -> Any:
        expr = expr.strip()
        if ":" in expr and expr.split(":", 1)[0] in _RESOLVERS:
            name, argstr = expr.split(":", 1)
            return _RESOLVERS[name](*_split_args(argstr))
        got = _lookup(root, expr)
        if isinstance(got, str) and "${" in got:
            got = _resolve_string(got, root, depth + 1)
        return got

    prev = None
    while "${" in value and value != prev:
        whole = _INTERP.fullmatch(value.strip())
        if whole is not None:
            return eval_expr(whole.group(1))  # keeps the native type of the target
        prev = value
        # innermost expressions first, so that "${a:${b}}" ends as one whole-value expression
        value = _INTERP.sub(lambda m: str(eval_expr(m.group(1))), value)
    return value


def resolve_interpolations(node: Any, root: Any = None) -> Any:
    root = node if root is None else root
    if isinstance(node, dict):
        return {k: resolve_interpolations(v, root) for k, v in node.items()}
    if isinstance(node, list):
        return [resolve_interpolations(v, root) for v in node]
    if isinstance(node, str) and "${" in node:
        return _resolve_string(node, root)
    return node


# ---------------------------------------------------------------------------------------------
# Schema-directed construction.
# ---------------------------------------------------------------------------------------------


def _type_name(tp: Any) -> str:
    return getattr(tp, "__name__", str(tp))


def _coerce(value: Any, tp: Any, where: str) -> Any:
    origin = typing.get_origin(tp)
    args = typing.get_args(tp)

    if tp is Any or tp is typing.Any:
        return value

    if origin is Union:
        if value is None and type(None) in args:
            return None
        errors = []
        # try exact-type matches first so that Union[int, str] keeps 5 an int and "2ep" a str
        for cand in args:
            if cand is type(None):
                continue
            if isinstance(cand, type) and type(value) is cand:
                return value
        for cand in args:
            if cand is type(None):
                continue
            try:
                return _coerce(value, cand, where)
            except OLMoConfigurationError as e:
                errors.append(str(e))
        raise OLMoConfigurationError(f"{where}: value {value!r} fits none of {tp}: {errors}")

    if value is None:
        raise OLMoConfigurationError(f"{where}: None is not allowed for type {_type_name(tp)}")

    if dataclasses.is_dataclass(tp):
        if isinstance(value, tp):
            return value
        if not isinstance(value, dict):
            raise OLMoConfigurationError(f"{where}: expected a mapping for {_type_name(tp)}, got {value!r}")
        return build(tp, value, where)

    if isinstance(tp, type) and issubclass(tp, Enum):
        if isinstance(value, tp):
            return value
        for member in tp:
            if value == member.value or value == member.name:
                return member
        if isinstance(value, str):
            for member in tp:
                if str(member.value).lower() == value.lower() or member.name.lower() == value.lower():
                    return member
        raise OLMoConfigurationError(
            f"{where}: {value!r} is not one of {[m.name for m in tp]} ({_type_name(tp)})"
        )

    if origin in (list, typing.List):
        if isinstance(value, tuple):
            value = list(value)
        if not isinstance(value, list):
            raise OLMoConfigurationError(f"{where}: expected a list, got {value!r}")
        elem = args[0] if args else Any
        return [_coerce(v, elem, f"{where}[{i}]") for i, v in enumerate(value)]

    if origin in (tuple, typing.Tuple):
        if not isinstance(value, (list, tuple)):
            raise OLMoConfigurationError(f"{where}: expected a sequence, got {value!r}")
        if len(args) == 2 and args[1] is Ellipsis:
            return tuple(_coerce(v, args[0], f"{where}[{i}]") for i, v in enumerate(value))
        if args and len(args) != len(value):
            raise OLMoConfigurationError(f"{where}: expected {len(args)} items, got {len(value)}")
        return tuple(_coerce(v, a, f"{where}[{i}]") for i, (v, a) in enumerate(zip(value, args or [Any] * len(value))))

    if origin in (dict, typing.Dict):
        if not isinstance(value, dict):
            raise OLMoConfigurationError(f"{where}: expected a mapping, got {value!r}")
        kt, vt = args if args else (Any, Any)
        return {_coerce(k, kt, f"{where}.<key>"): _coerce(v, vt, f"{where}.{k}") for k, v in value.items()}

    if tp is bool:
        if isinstance(value, bool):
            return value
        if isinstance(value, str) and value.lower() in ("true", "false", "yes", "no", "on", "off", "1", "0"):
            return value.lower() in ("true", "yes", "on", "1")
        if isinstance(value, int) and value in (0, 1):
            return bool(value)
        raise OLMoConfigurationError(f"{where}: {value!r} is not a bool")

    if tp is int:
        if isinstance(value, bool):
            raise OLMoConfigurationError(f"{where}: {value!r} is not an int")
        if isinstance(value, int):
            return value
        if isinstance(value, float) and value.is_integer():
            return int(value)
        if isinstance(value, str):
            try:
                return int(value.replace("_", ""))
            except ValueError:
                pass
        raise OLMoConfigurationError(f"{where}: {value!r} is not an int")

    if tp is float:
        if isinstance(value, bool):
            raise OLMoConfigurationError(f"{where}: {value!r} is not a float")
        if isinstance(value, (int, float)):
            return float(value)
        if isinstance(value, str):
            try:
                return float(value)
            except ValueError:
                pass
        raise OLMoConfigurationError(f"{where}: {value!r} is not a float")

    if tp is str:
        if isinstance(value, Enum):
            return str(value.value)
        if isinstance(value, (str, int, float, bool)):
            return str(value) if not isinstance(value, str) else value
        raise OLMoConfigurationError(f"{where}: {value!r} is not a string")

    if isinstance(tp, type) and isinstance(value, tp):
        return value
    raise OLMoConfigurationError(f"{where}: cannot interpret {value!r} as {_type_name(tp)}")


def _hints(cls: Type) -> Dict[str, Any]:
    import sys

    mod = sys.modules.get(cls.__module__)
    ns = dict(vars(mod)) if mod is not None else {}
    return typing.get_type_hints(cls, globalns=ns)


def build(cls: Type, data: Optional[Dict[str, Any]] = None, where: str = "") -> Any:
    """Instantiate dataclass ``cls`` from a plain mapping, validating and coercing every field."""
    data = {} if data is None else data
    if not dataclasses.is_dataclass(cls):
        raise TypeError(f"{cls} is not a dataclass")
    hints = _hints(cls)
    fields = {f.name: f for f in dataclasses.fields(cls) if f.init}
    unknown = [k for k in data if k not in fields]
    if unknown:
        import difflib

        prefix = f"{where}." if where else ""
        near = difflib.get_close_matches(str(unknown[0]), list(fields), n=2, cutoff=0.7)
        raise OLMoConfigurationError(
            f"Key '{prefix}{unknown[0]}' is not in struct {cls.__name__}"
            + (f" (also: {unknown[1:]})" if len(unknown) > 1 else "")
            + (f"; did you mean {' or '.join(repr(prefix + n) for n in near)}?" if near else "")
        )
    kwargs: Dict[str, Any] = {}
    for name, f in fields.items():
        path = f"{where}.{name}" if where else name
        if name in data:
            kwargs[name] = _coerce(data[name], hints[name], path)
        elif f.default is dataclasses.MISSING and f.default_factory is dataclasses.MISSING:  # type: ignore
            raise OLMoConfigurationError(f"Missing mandatory value: {path}")
    return cls(**kwargs)


def to_container(obj: Any, enum_to_str: bool = True) -> Any:
    """Dataclass tree -> plain dict/list tree suitable for YAML or ``wandb.config``."""
    if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        return {f.name: to_container(getattr(obj, f.name), enum_to_str) for f in dataclasses.fields(obj)}
    if isinstance(obj, Enum):
        return obj.name if enum_to_str else obj
    if isinstance(obj, dict):
        return {k: to_container(v, enum_to_str) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [to_container(v, enum_to_str) for v in obj]
    return obj
