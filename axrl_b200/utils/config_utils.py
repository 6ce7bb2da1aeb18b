"""Config loading: YAML file < ``--a.b=v`` CLI flags < ``AXRL__a__b=v`` env vars.

Behaviour follows reference ``axrl/utils/config_utils.py:107-189`` (merge
order, ``config_path`` override from CLI/env, strict validation, torch-dtype
string round trip).  The dotted-key merge is implemented here directly
(no OmegaConf dependency): each value string is parsed as a YAML scalar/list
so ``true``/``null``/``[1,2]``/``1e-5`` get their natural types.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path
from typing import Any

import yaml
from pydantic import ValidationError

from axrl_b200.configs import StrictBaseModel

ENV_CONFIG_PREFIX = "AXRL__"

_DTYPE_NAMES = ("float32", "float16", "bfloat16", "int32", "int64", "uint8", "bool")


def _parse_scalar(text: str) -> Any:
    try:
        value = yaml.safe_load(text)
    except yaml.YAMLError:
        return text
    # YAML reads "1e-5" as a string; accept plain floats too.
    if isinstance(value, str):
        try:
            return float(value) if any(c in value for c in ".eE") else value
        except ValueError:
            return value
    return value


def _set_dotted(tree: dict, dotted: str, value: Any) -> None:
    keys = dotted.split(".")
    node = tree
    for k in keys[:-1]:
        nxt = node.get(k)
        if not isinstance(nxt, dict):
            nxt = {}
            node[k] = nxt
        node = nxt
    node[keys[-1]] = value


def _deep_merge(base: dict, over: dict) -> dict:
    out = dict(base)
    for k, v in over.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = _deep_merge(out[k], v)
        else:
            out[k] = v
    return out


def parse_cli_overrides(argv: list[str]) -> dict:
    """``--a.b=1 --c=x`` (also ``a.b=1``) -> nested dict."""
    tree: dict = {}
    for arg in argv:
        if "=" not in arg:
            continue
        key, raw = arg.split("=", 1)
        _set_dotted(tree, key.lstrip("-"), _parse_scalar(raw))
    return tree


def load_env_overrides(prefix: str = ENV_CONFIG_PREFIX, environ: dict[str, str] | None = None) -> dict:
    environ = os.environ if environ is None else environ
    tree: dict = {}
    for key in sorted(environ):
        if key.startswith(prefix) and len(key) > len(prefix):
            _set_dotted(tree, key[len(prefix):].replace("__", "."), _parse_scalar(environ[key]))
    return tree


def _dtypes_to_str(obj: Any) -> Any:
    if type(obj).__module__ == "torch" and type(obj).__qualname__ == "dtype":
        return str(obj)
    if isinstance(obj, dict):
        return {k: _dtypes_to_str(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_dtypes_to_str(v) for v in obj]
    return obj


def _str_to_dtypes(obj: Any) -> Any:
    if isinstance(obj, str) and obj.startswith("torch.") and obj[6:] in _DTYPE_NAMES:
        import torch

        return getattr(torch, obj[6:])
    if isinstance(obj, dict):
        return {k: _str_to_dtypes(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_str_to_dtypes(v) for v in obj]
    return obj


def _flatten(d: dict, prefix: str = "") -> dict[str, Any]:
    out: dict[str, Any] = {}
    for k, v in d.items():
        key = f"{prefix}.{k}" if prefix else k
        if isinstance(v, dict):
            out.update(_flatten(v, key))
        else:
            out[key] = v
    return out


def _fmt(v: Any) -> str:
    if v is None:
        return "null"
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, list):
        return "[" + ",".join(_fmt(x) for x in v) + "]"
    return str(v)


def config_to_args(config: StrictBaseModel) -> dict[str, str]:
    """Flatten a config into sorted ``{"--a.b": "v"}`` CLI-style pairs."""
    flat = _flatten(_dtypes_to_str(config.model_dump()))
    return {f"--{k}": _fmt(v) for k, v in sorted(flat.items())}


def save_to_yaml(config: StrictBaseModel, path: Path) -> None:
    with Path(path).open("w") as f:
        yaml.safe_dump(_dtypes_to_str(config.model_dump()), f, sort_keys=False, indent=4)


def load_and_validate_config[T: StrictBaseModel](
    config_class: type[T],
    config_path: str | None = None,
    *,
    load_env_config: bool = True,
    print_configs: bool = False,
    argv: list[str] | None = None,
) -> T:
    """Merge YAML < CLI < env and validate strictly against ``config_class``."""
    cli = parse_cli_overrides(sys.argv[1:] if argv is None else argv)
    env = load_env_overrides() if load_env_config else {}
    if "config_path" in cli:
        config_path = cli.pop("config_path")
    if "config_path" in env:
        config_path = env.pop("config_path")
    base: dict = {}
    if config_path:
        with open(config_path) as f:
            base = yaml.safe_load(f) or {}
    merged = _str_to_dtypes(_deep_merge(_deep_merge(base, cli), env))
    try:
        cfg = config_class.model_validate(merged, strict=True)
    except ValidationError as e:
        for err in e.errors():
            print(f"config error at {'.'.join(str(x) for x in err['loc'])}: {err['msg']}", file=sys.stderr)
        raise ValueError("Configuration validation failed") from None
    if print_configs:
        print(cfg)
    return cfg
