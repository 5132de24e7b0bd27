"""Model catalog: entries from the presets (sizes from the configs), name resolution from the
spellings users type, suggestions for unknown names, the user catalog file, and `squish pull`
through the catalog."""
import json

import pytest

from squish_b200 import catalog as C


@pytest.fixture()
def home(tmp_path, monkeypatch):
    monkeypatch.setenv("SQUISH_HOME", str(tmp_path / "home"))
    monkeypatch.delenv("SQUISH_CONFIG_DIR", raising=False)
    (tmp_path / "home").mkdir()
    return tmp_path / "home"


def test_entries_sizes_and_order(home):
    es = C.list_catalog()
    assert [e.params_b for e in es] == sorted(e.params_b for e in es)
    e7 = C.resolve("qwen2.5:7b")
    assert e7.preset == "qwen2.5-7b" and 7.0 < e7.params_b < 8.0
    assert e7.int4_size_gb < e7.size_gb / 2.5  # INT4 codes + scales vs bf16
    moe = C.resolve("qwen3:30b-a3b")
    assert moe.moe and 2.5 < moe.active_params_b < 4.0 and "moe" in moe.tags
    assert [e.id for e in C.list_catalog("moe")] == ["qwen3:30b-a3b"]


@pytest.mark.parametrize("name,want", [("Qwen/Qwen2.5-7B-Instruct", "qwen2.5:7b"), ("qwen2.5-7b-int4", "qwen2.5:7b"),
                                       ("qwen3-30b-a3b", "qwen3:30b-a3b"), ("Llama-3.1-8B-Instruct", "llama3.1:8b"),
                                       ("llama-3-70b", "llama3:70b"), ("QWEN3:8B", "qwen3:8b"),
                                       ("meta-llama/Meta-Llama-3-70B-Instruct", "llama3:70b")])
def test_resolve_spellings(home, name, want):
    assert C.resolve(name).id == want


def test_unknown_names_get_suggestions(home):
    assert C.resolve("qwen3") is None and C.resolve("mistral:7b") is None
    assert C.suggest("qwen7b")[0].id == "qwen2.5:7b"
    assert C.suggest("llama 70")[0].id == "llama3:70b"
    assert C.suggest("zzz") == []
    assert {e.id for e in C.search("reasoning")} == {"qwen3:8b", "qwen3:30b-a3b"}


def test_user_catalog_adds_and_overrides(home):
    (home / "catalog.json").write_text(json.dumps([
        {"id": "qwen2.5:7b", "notes": "local build"},
        {"id": "tiny:1m", "name": "Tiny test model", "hf_repo": "local/tiny", "params": "1M", "params_b": 0.001,
         "context": 2048, "size_gb": 0.0, "int4_size_gb": 0.0, "preset": "tiny-llama", "tags": ["test"]}]))
    cat = C.load_catalog()
    assert cat["qwen2.5:7b"].notes == "local build" and cat["qwen2.5:7b"].preset == "qwen2.5-7b"
    assert C.resolve("tiny-1m").preset == "tiny-llama"


def test_pull_through_the_catalog(home, capsys):
    from squish_b200.cli import main

    (home / "catalog.json").write_text(json.dumps([
        {"id": "tiny:1m", "name": "Tiny", "hf_repo": "local/tiny", "params": "1M", "params_b": 0.001, "context": 2048,
         "size_gb": 0.0, "int4_size_gb": 0.0, "preset": "tiny-llama"}]))
    assert main(["pull", "qwen7"]) == 2
    assert "did you mean" in capsys.readouterr().err
    assert main(["pull", "tiny:1m", "--device", "cpu"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["n_quantized"] > 0 and (home / "models" / "tiny-llama" / "tensors").is_dir()
