"""YAML config loading with the reference schema and its interpolations.

The reference loads its YAML through LightX2V/OmegaConf
(``configs/minimax_h3_t2av_dmd_a100_world16.yaml:1-144``) and relies on two
resolvers: ``${oc.env:VAR,default}`` and ``${oc.decode:...}``.  OmegaConf is not
a dependency here, so this module implements exactly those resolvers plus plain
``${a.b.c}`` node references, innermost first, on ordinary dicts.

Schema additions (all optional, so the reference YAMLs load unchanged):

* ``training.b200`` is accepted as an alias of ``training.a100``;
* ``synthetic:`` gives the DiT dims, token counts and seeds used in place of
  ``pretrained_model_name_or_path`` / ``data_path``;
* ``kernels: {backend: native|torch}`` picks, once at build time, the
  hand-written sm_100a kernels or the PyTorch (cuBLAS + SDPA) path.
"""

from __future__ import annotations

import copy
import os
import re
from pathlib import Path
from typing import Any

import yaml

_INTERP = re.compile(r"\$\{([^${}]*)\}")


class ConfigError(ValueError):
    pass


def _lookup(root: dict[str, Any], dotted: str) -> Any:
    node: Any = root
    for part in dotted.split("."):
        if not isinstance(node, dict) or part not in node:
            raise ConfigError(f"interpolation references missing key {dotted!r}")
        node = node[part]
    return node


def _resolve_expr(expr: str, root: dict[str, Any]) -> Any:
    expr = expr.strip()
    if expr.startswith("oc.env:"):
        body = expr[len("oc.env:"):]
        name, _, default = body.partition(",")
        value = os.environ.get(name.strip())
        if value is None:
            if not _:
                raise ConfigError(f"environment variable {name.strip()!r} is not set and has no default")
            return default.strip()
        return value
    if expr.startswith("oc.decode:"):
        return yaml.safe_load(expr[len("oc.decode:"):])
    return _lookup(root, expr)


def _resolve_string(text: str, root: dict[str, Any], depth: int = 0) -> Any:
    if depth > 32:
        raise ConfigError(f"interpolation too deep in {text!r}")
    match = _INTERP.search(text)
    if match is None:
        return text
    value = _resolve_expr(match.group(1), root)
    if match.span() == (0, len(text)):
        # Whole-string interpolation keeps the resolved type (int, float, ...).
        if isinstance(value, str) and "${" in value:
            return _resolve_string(value, root, depth + 1)
        return value
    rebuilt = text[: match.start()] + str(value) + text[match.end():]
    return _resolve_string(rebuilt, root, depth + 1)


def _resolve_tree(node: Any, root: dict[str, Any]) -> Any:
    if isinstance(node, dict):
        return {key: _resolve_tree(value, root) for key, value in node.items()}
    if isinstance(node, list):
        return [_resolve_tree(value, root) for value in node]
    if isinstance(node, str) and "${" in node:
        return _resolve_string(node, root)
    return node


def resolve(config: dict[str, Any]) -> dict[str, Any]:
    """Resolve every interpolation in ``config`` (returns a new dict)."""
    raw = copy.deepcopy(config)
    return _resolve_tree(raw, raw)


def training_system_section(config: dict[str, Any]) -> dict[str, Any]:
    """Return ``training.a100`` (reference name) or its alias ``training.b200``."""
    training = config.get("training", {}) or {}
    if "a100" in training and "b200" in training:
        raise ConfigError("set only one of training.a100 and training.b200")
    return training.get("a100", training.get("b200", {})) or {}


def load_config(path: str | os.PathLike[str], overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    """Load, merge ``overrides`` (nested dict) and resolve a YAML config."""
    text = Path(path).read_text(encoding="utf-8")
    config = yaml.safe_load(text) or {}
    if not isinstance(config, dict):
        raise ConfigError(f"{path}: top level must be a mapping")
    if overrides:
        config = merge(config, overrides)
    config = resolve(config)
    config.setdefault("_meta", {})["path"] = str(path)
    return config


def merge(base: dict[str, Any], override: dict[str, Any]) -> dict[str, Any]:
    out = copy.deepcopy(base)
    for key, value in override.items():
        if isinstance(value, dict) and isinstance(out.get(key), dict):
            out[key] = merge(out[key], value)
        else:
            out[key] = copy.deepcopy(value)
    return out


def get(config: dict[str, Any], dotted: str, default: Any = None) -> Any:
    node: Any = config
    for part in dotted.split("."):
        if not isinstance(node, dict) or part not in node:
            return default
        node = node[part]
    return node


def env_flag(name: str, default: bool) -> bool:
    value = os.environ.get(name)
    if value is None:
        return bool(default)
    return value.strip().lower() in {"1", "true", "yes", "on"}
