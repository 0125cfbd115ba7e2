"""Config registry for the plugins -- same mechanism and schema as the
reference's ``kernel_configs/__init__.py:60-111``: every ``<name>.toml`` in this directory is
parsed and merged with the callables of its companion ``<name>.py`` (``input_generator``,
``reference_fn``, ``flops_fn``, ``bytes_fn`` and the optional ``numerical_stability_cases``,
``optimization_traits``, ``KERNEL_OPT_CHARACTERISTICS``) into ``KERNEL_CONFIGS[name]``."""

from __future__ import annotations

import importlib
import pathlib
import tomllib
from typing import Any, Dict

from ._utils import DTYPE_MAP

_PKG_DIR = pathlib.Path(__file__).resolve().parent


def _sizes(raw: list[dict]) -> list[tuple[str, dict]]:
    return [(entry["label"], dict(entry["params"])) for entry in raw]


def _dtypes(raw: list[str]):
    unknown = [n for n in raw if n not in DTYPE_MAP]
    if unknown:
        raise ValueError(f"Unknown dtype strings {unknown}. Valid: {list(DTYPE_MAP)}")
    return [DTYPE_MAP[n] for n in raw]


def _tolerances(raw: dict):
    out = {}
    for name, tol in raw.items():
        if name not in DTYPE_MAP:
            raise ValueError(f"Unknown dtype '{name}' in tolerances section")
        out[DTYPE_MAP[name]] = {"atol": float(tol["atol"]), "rtol": float(tol["rtol"])}
    return out


def _build_config(toml_path: pathlib.Path) -> Dict[str, Any]:
    with open(toml_path, "rb") as f:
        data = tomllib.load(f)
    mod = importlib.import_module(f"{__name__}.{toml_path.stem}")
    meta = data.get("meta", {})
    cfg: Dict[str, Any] = {"meta": meta}
    if meta.get("multi_output", False):
        cfg["multi_output"] = True
    cfg["test_sizes"] = _sizes(data["test_sizes"])
    raw_dtypes = data.get("test_dtypes", meta.get("test_dtypes"))
    if raw_dtypes is None:
        raise KeyError("test_dtypes")
    cfg["test_dtypes"] = _dtypes(raw_dtypes)
    cfg["tolerances"] = _tolerances(data["tolerances"])
    cfg["edge_sizes"] = _sizes(data.get("edge_sizes", []))
    for key in ("input_generator", "reference_fn", "flops_fn", "bytes_fn"):
        cfg[key] = getattr(mod, key)
    for attr, key in (("numerical_stability_cases", "numerical_stability_cases"),
                      ("optimization_traits", "optimization_traits"),
                      ("KERNEL_OPT_CHARACTERISTICS", "kernel_opt_characteristics")):
        if hasattr(mod, attr):
            cfg[key] = getattr(mod, attr)
    return cfg


def _discover() -> Dict[str, Dict[str, Any]]:
    configs: Dict[str, Dict[str, Any]] = {}
    for toml_path in sorted(_PKG_DIR.glob("*.toml")):
        if not toml_path.with_suffix(".py").exists():
            raise FileNotFoundError(f"Kernel config '{toml_path.name}' has no companion .py")
        configs[toml_path.stem] = _build_config(toml_path)
    return configs


KERNEL_CONFIGS: Dict[str, Dict[str, Any]] = _discover()
