"""Minimal stand-in for the ``omegaconf`` package, used only by the reference arm of bench.py.

The image has no ``omegaconf`` wheel and no network. The reference framework
imports it at module import time (its config module builds a structured
default tree from dataclasses); its training loop itself only reads plain
mappings. This stand-in implements exactly the calls that path makes:
``OmegaConf.structured``, ``OmegaConf.to_container``, ``OmegaConf.create``,
``OmegaConf.merge``, ``OmegaConf.load``, ``OmegaConf.set_struct``,
``OmegaConf.resolve`` and the ``DictConfig`` type. It is not part of the
koochak_b200 package and never touches the benchmark's hot path.
"""

from __future__ import annotations

import copy
import dataclasses
from typing import Any, Mapping


class DictConfig(dict):
    def __getattr__(self, name):
        try:
            return self[name]
        except KeyError:
            raise AttributeError(name) from None

    def __setattr__(self, name, value):
        self[name] = value


class ListConfig(list):
    pass


def _to_node(v: Any) -> Any:
    if dataclasses.is_dataclass(v):
        return DictConfig({f.name: _to_node(getattr(v, f.name)) for f in dataclasses.fields(v)})
    if isinstance(v, Mapping):
        return DictConfig({k: _to_node(x) for k, x in v.items()})
    if isinstance(v, (list, tuple)):
        return ListConfig(_to_node(x) for x in v)
    return v


def _plain(v: Any) -> Any:
    if isinstance(v, Mapping):
        return {k: _plain(x) for k, x in v.items()}
    if isinstance(v, list):
        return [_plain(x) for x in v]
    return v


class OmegaConf:
    @staticmethod
    def structured(obj: Any) -> DictConfig:
        if isinstance(obj, type) and dataclasses.is_dataclass(obj):
            obj = obj()
        return _to_node(obj)

    @staticmethod
    def create(obj: Any = None) -> DictConfig:
        return _to_node(obj or {})

    @staticmethod
    def to_container(cfg: Any, resolve: bool = False) -> Any:
        return _plain(cfg)

    @staticmethod
    def merge(*cfgs: Any) -> DictConfig:
        out: dict = {}

        def into(dst: dict, src: Mapping) -> None:
            for k, v in src.items():
                if isinstance(v, Mapping) and isinstance(dst.get(k), Mapping):
                    into(dst[k], v)
                else:
                    dst[k] = copy.deepcopy(_plain(v))

        for c in cfgs:
            into(out, _plain(_to_node(c)))
        return _to_node(out)

    @staticmethod
    def load(path: str) -> DictConfig:
        import yaml

        with open(path, encoding="utf-8") as fh:
            return _to_node(yaml.safe_load(fh) or {})

    @staticmethod
    def set_struct(cfg: Any, value: bool) -> None:
        return None

    @staticmethod
    def resolve(cfg: Any) -> None:
        return None
