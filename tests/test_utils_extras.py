"""Environment lookups, structured logging, CSV / INI / JSON helpers and counter sets."""
import json

import pytest

from brain_b200.utils import extras as U


def test_env_helpers(monkeypatch):
    monkeypatch.setenv("BRX_N", "42")
    monkeypatch.setenv("BRX_F", "2.5")
    monkeypatch.setenv("BRX_B", "Yes")
    monkeypatch.setenv("BRX_BAD", "maybe")
    monkeypatch.setenv("BRX_L", " a, b ,,c ")
    assert U.env_i64("BRX_N", 0) == 42 and U.env_i64("BRX_F", 7) == 7 and U.env_f64("BRX_F", 0) == 2.5
    assert U.env_bool("BRX_B", False) and U.env_bool("BRX_BAD", True) and not U.env_bool("BRX_MISSING", False)
    assert U.env_list("BRX_L") == ["a", "b", "c"] and U.env_list("BRX_MISSING") == []
    assert U.env_get_or("BRX_MISSING", "d") == "d"
    m = U.env_prefix_map("BRX_")
    assert m["n"] == "42" and list(m) == sorted(m)
    pe = U.PrefixEnv("BRX_")
    assert pe.get("N") == "42" and pe.get_i64("n", 0) == 42 and pe.get_bool("b", False)


def test_structured_logger():
    sink = U.MemorySink()
    lg = U.StandardLogger(U.LogLevel.from_str("warning"), sink, U.KeyValueFormatter())
    assert not lg.info("net", "skipped")
    assert lg.error("net", 'bad "frame"', peer=3)
    assert sink.get_messages() == ['level=ERROR target=net msg="bad \\"frame\\"" peer="3"']
    multi = U.MultiSink([sink])
    m2 = U.MemorySink()
    multi.add_sink(m2)
    rec = U.create_record(U.LogLevel.WARN, "io", "slow").with_location("a.rs", 7).with_field("ms", 12)
    U.StandardLogger(U.LogLevel.TRACE, multi, U.JsonLogFormatter()).log(rec)
    d = json.loads(m2.get_messages()[0])
    assert d["level"] == "WARN" and d["file"] == "a.rs" and d["line"] == 7 and d["fields"] == {"ms": "12"}
    assert U.PlainFormatter().format(rec) == "[WARN] [io] slow"
    assert "(a.rs:7)" in U.TimestampedFormatter().format(rec)
    assert U.LogLevel.from_str("bogus") == U.LogLevel.INFO
    assert not U.StandardLogger(U.LogLevel.OFF, sink).error("x", "y")


def test_csv_ini_json_counters(tmp_path):
    r = U.CsvReader.parse_str('name,quote\nada,"said ""hi"", then left"\nbob,plain\n')
    assert r.headers() == ["name", "quote"] and r.records()[0].get(1) == 'said "hi", then left'
    assert r.records()[1].get(5) is None
    with pytest.raises(ValueError):
        U.CsvReader.parse_str('a,"open\n')
    w = U.CsvWriter(U.CsvConfig(delimiter=";"))
    w.write_record(["x", "a;b", 3])
    assert w.to_string() == 'x;"a;b";3\n'
    ini = U.IniFile.parse("; c\n[train]\nlr = 0.1\nsteps=100\nfused = on\n")
    assert ini.get_f64("train", "lr") == 0.1 and ini.get_i64("train", "steps") == 100
    assert ini.get_bool("train", "fused") and ini.get_i64("train", "missing", 5) == 5
    assert U.IniFile.parse(ini.to_string()).sections == ini.sections
    j = U.JsonValue.parse('{"a": [1, 2.5, true], "s": "t", "n": null}')
    assert j.get("a").as_array()[1].as_f64() == 2.5 and j.get("a").get(2).as_bool() is True
    assert j.get("a").get(0).as_bool() is None and j.get("s").as_str() == "t" and j.get("n").is_null()
    assert j.to_compact_string() == '{"a":[1,2.5,true],"s":"t","n":null}'
    cs = U.CounterSet()
    cs.increment("b")
    cs.increment("a", 3)
    cs.get_gauge("load").set(0.5)
    assert cs.snapshot_counters() == {"a": 3, "b": 1} and cs.snapshot_gauges() == {"load": 0.5}
    cs.reset_all()
    assert cs.snapshot_counters() == {} and cs.get_gauge("load").get() == 0.0
    p = tmp_path / "f.txt"
    p.write_text("hey")
    assert U.read_file_str(str(p)) == "hey" and U.read_file_bytes(str(p)) == b"hey"
    assert U.delete_file(str(p)) and not U.delete_file(str(p))
