"""Small text-format helpers: INI, JSON and CSV read / write with typed values.

Reference: crates/brain-utils (JSON / CSV / INI parsers, config/mod.rs:55 ``ConfigManager`` sources).
INI values are typed on read: ``true/false`` -> bool, integers, floats, otherwise strings.
"""
from __future__ import annotations

import configparser
import csv
import io
import json


def _typed(v: str):
    s = v.strip()
    if s.lower() in ("true", "yes", "on"):
        return True
    if s.lower() in ("false", "no", "off"):
        return False
    for cast in (int, float):
        try:
            return cast(s)
        except ValueError:
            pass
    return s


def parse_ini(text: str) -> dict:
    """{section: {key: typed value}}; keys before any section go to "" (the default section)."""
    cp = configparser.ConfigParser(interpolation=None, default_section="\0")
    cp.optionxform = str
    cp.read_string("[\0root]\n" + text)
    out = {}
    for sec in cp.sections():
        out["" if sec == "\0root" else sec] = {k: _typed(v) for k, v in cp.items(sec)}
    if not out.get(""):
        out.pop("", None)
    return out


def dump_ini(data: dict) -> str:
    lines = []
    for k, v in data.get("", {}).items():
        lines.append(f"{k} = {str(v).lower() if isinstance(v, bool) else v}")
    for sec, kv in data.items():
        if sec == "":
            continue
        lines.append(f"[{sec}]")
        lines += [f"{k} = {str(v).lower() if isinstance(v, bool) else v}" for k, v in kv.items()]
    return "\n".join(lines) + "\n"


def parse_json(text: str):
    return json.loads(text)


def dump_json(obj, indent: int | None = 1) -> str:
    return json.dumps(obj, indent=indent, sort_keys=True)


def parse_csv(text: str, header: bool = True, typed: bool = True):
    """Rows as dicts (with a header) or lists; values typed like INI values."""
    rows = list(csv.reader(io.StringIO(text)))
    conv = (lambda r: [_typed(v) for v in r]) if typed else (lambda r: r)
    if not header:
        return [conv(r) for r in rows if r]
    head = rows[0]
    return [dict(zip(head, conv(r))) for r in rows[1:] if r]


def dump_csv(rows, header=None) -> str:
    buf = io.StringIO()
    w = csv.writer(buf, lineterminator="\n")
    if rows and isinstance(rows[0], dict):
        header = header or list(rows[0])
        w.writerow(header)
        w.writerows([[r.get(h, "") for h in header] for r in rows])
    else:
        if header:
            w.writerow(header)
        w.writerows(rows)
    return buf.getvalue()
