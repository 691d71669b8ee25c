"""Configuration helpers (reference brain-utils ConfigManager with source precedence and
EnvConfig::from_prefix; crates/brain-utils/src/config/mod.rs:55, env.rs:68).

Precedence (highest first): values set with ``force_set`` > environment (``BRAIN_*`` by default) >
values set with ``set`` (e.g. from a config file) > defaults. ``load_file`` reads JSON or YAML.
"""
from __future__ import annotations

import json
import os


def _coerce(v: str):
    for f in (int, float):
        try:
            return f(v)
        except ValueError:
            pass
    if v.lower() in ("true", "false"):
        return v.lower() == "true"
    return v


class EnvConfig:
    def __init__(self, values: dict):
        self.values = values

    @staticmethod
    def from_prefix(prefix: str = "BRAIN_") -> "EnvConfig":
        return EnvConfig({k[len(prefix):].lower(): _coerce(v) for k, v in os.environ.items() if k.startswith(prefix)})

    def get(self, key, default=None):
        return self.values.get(key.lower(), default)


class ConfigManager:
    def __init__(self, defaults: dict | None = None, env_prefix: str = "BRAIN_"):
        self.defaults = dict(defaults or {})
        self.file: dict = {}
        self.forced: dict = {}
        self.env_prefix = env_prefix

    def set(self, key, value) -> None:
        self.file[key] = value

    def force_set(self, key, value) -> None:
        self.forced[key] = value

    def load_file(self, path: str) -> None:
        with open(path) as f:
            text = f.read()
        if path.endswith((".yaml", ".yml")):
            import yaml
            data = yaml.safe_load(text) or {}
        else:
            data = json.loads(text)
        self.file.update(data)

    def get(self, key, default=None):
        if key in self.forced:
            return self.forced[key]
        env = os.environ.get(self.env_prefix + key.upper())
        if env is not None:
            return _coerce(env)
        if key in self.file:
            return self.file[key]
        return self.defaults.get(key, default)

    def as_dict(self) -> dict:
        keys = set(self.defaults) | set(self.file) | set(self.forced)
        return {k: self.get(k) for k in sorted(keys)}
