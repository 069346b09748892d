"""JSON-serialisable dataclass configs (the reference's ``config/base_config.py:15-219``
interface: ``to_dict / to_json / from_dict / from_json / update / merge / validate``,
``load_config / save_config / merge_configs / create_config_from_args / get_config_diff``).

Nested dataclass fields, tuples and enums survive a round trip: ``from_dict`` rebuilds a
nested dataclass from its dict, a tuple field from its list and an ``Enum`` field (or a
list of them) from its values.
"""
from __future__ import annotations

import dataclasses
import enum
import json
import typing
from pathlib import Path
from typing import Any, Dict, Type, TypeVar

T = TypeVar("T", bound="BaseConfig")


def _encode(v: Any) -> Any:
    if isinstance(v, enum.Enum):
        return v.value
    if dataclasses.is_dataclass(v):
        return {f.name: _encode(getattr(v, f.name)) for f in dataclasses.fields(v)}
    if isinstance(v, (list, tuple)):
        return [_encode(x) for x in v]
    if isinstance(v, dict):
        return {k: _encode(x) for k, x in v.items()}
    return v


def _decode(tp: Any, v: Any) -> Any:
    """Rebuild ``v`` (from JSON) as type ``tp`` where the annotation says how."""
    if v is None:
        return None
    origin = typing.get_origin(tp)
    args = typing.get_args(tp)
    if origin is typing.Union:
        for a in args:
            if a is type(None):
                continue
            try:
                return _decode(a, v)
            except (TypeError, ValueError):
                continue
        return v
    if isinstance(tp, type) and issubclass(tp, enum.Enum):
        return tp(v) if not isinstance(v, tp) else v
    if isinstance(tp, type) and dataclasses.is_dataclass(tp) and isinstance(v, dict):
        return _from_dict(tp, v)
    if origin in (list, typing.List) and args and isinstance(v, (list, tuple)):
        return [_decode(args[0], x) for x in v]
    if origin in (tuple, typing.Tuple) and isinstance(v, (list, tuple)):
        return tuple(v)
    return v


def _from_dict(cls, d: Dict[str, Any]):
    hints = typing.get_type_hints(cls)
    names = {f.name for f in dataclasses.fields(cls) if f.init}
    kw = {k: _decode(hints.get(k, Any), v) for k, v in d.items() if k in names}
    return cls(**kw)


class BaseConfig:
    """Mixin for ``@dataclass`` configs."""

    def to_dict(self) -> Dict[str, Any]:
        return _encode(self)

    def to_json(self, filepath: str | None = None) -> str:
        s = json.dumps(self.to_dict(), indent=2, sort_keys=True)
        if filepath:
            Path(filepath).parent.mkdir(parents=True, exist_ok=True)
            Path(filepath).write_text(s)
        return s

    @classmethod
    def from_dict(cls: Type[T], config_dict: Dict[str, Any]) -> T:
        return _from_dict(cls, config_dict)

    @classmethod
    def from_json(cls: Type[T], json_str_or_path: str) -> T:
        p = Path(json_str_or_path)
        try:
            is_file = p.exists()
        except OSError:          # a long JSON string is not a path
            is_file = False
        return cls.from_dict(json.loads(p.read_text() if is_file else json_str_or_path))

    def update(self, **kwargs) -> None:
        for k, v in kwargs.items():
            if not hasattr(self, k):
                raise ValueError(f"Invalid config key: {k}")
            setattr(self, k, v)

    def merge(self: T, other: T) -> T:
        """A new config: this one's values overridden by ``other``'s non-None ones."""
        a, b = self.to_dict(), other.to_dict()
        a.update({k: v for k, v in b.items() if v is not None})
        return self.__class__.from_dict(a)

    def validate(self) -> None:
        pass

    def __post_init__(self):
        self.validate()


def load_config(config_class: Type[T], config_path: str) -> T:
    return config_class.from_json(config_path)


def save_config(config: BaseConfig, config_path: str) -> None:
    config.to_json(config_path)


def merge_configs(*configs: BaseConfig) -> BaseConfig:
    if not configs:
        raise ValueError("At least one config must be provided")
    out = configs[0]
    for c in configs[1:]:
        out = out.merge(c)
    return out


def create_config_from_args(config_class: Type[T], args_dict: Any) -> T:
    if hasattr(args_dict, "__dict__") and not isinstance(args_dict, dict):
        args_dict = vars(args_dict)
    return config_class.from_dict({k: v for k, v in args_dict.items() if v is not None})


def get_config_diff(config1: BaseConfig, config2: BaseConfig) -> Dict[str, tuple]:
    a, b = config1.to_dict(), config2.to_dict()
    return {k: (a.get(k), b.get(k)) for k in sorted(set(a) | set(b)) if a.get(k) != b.get(k)}
