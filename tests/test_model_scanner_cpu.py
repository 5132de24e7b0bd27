"""Pre-load safety scan, local model discovery and the startup report."""
import json
import pickle

import numpy as np
import pytest
import torch


class _Evil:
    def __reduce__(self):
        import os

        return (os.getcwd, ())  # harmless if ever run; the scan must flag the import regardless


def test_scan_flags_code_importing_pickles_and_object_npy(tmp_path):
    from squish_b200.serving.model_scanner import scan_before_load

    torch.save({"w": torch.ones(3)}, tmp_path / "ok.pt")
    np.save(tmp_path / "ok.npy", np.arange(4, dtype=np.float32))
    (tmp_path / "ok.gguf").write_bytes(b"GGUF" + bytes(20))
    from safetensors.torch import save_file

    save_file({"a": torch.zeros(2, 2)}, str(tmp_path / "ok.safetensors"))
    r = scan_before_load(tmp_path)
    assert r.status == "clean" and r.scanned == 4, r.findings

    (tmp_path / "evil.pkl").write_bytes(pickle.dumps(_Evil()))
    np.save(tmp_path / "obj.npy", np.array([{"a": 1}], dtype=object), allow_pickle=True)
    (tmp_path / "bad.gguf").write_bytes(b"GGML" + bytes(20))
    (tmp_path / "bad.safetensors").write_bytes((10 ** 9).to_bytes(8, "little") + b"{}")
    r = scan_before_load(tmp_path)
    assert r.status == "unsafe"
    text = "\n".join(r.findings)
    for name in ("evil.pkl", "obj.npy", "bad.gguf", "bad.safetensors"):
        assert name in text
    assert "ok.pt" not in text


def test_loader_refuses_unsafe_checkpoints(tmp_path, monkeypatch):
    from squish_b200.io.convert import compress, load_checkpoint

    out = tmp_path / "m"
    compress(None, str(out), random_preset="tiny-llama", device="cpu", log=lambda *_: None)
    load_checkpoint(str(out), "cpu")  # clean
    np.save(out / "tensors" / "x__pt.npy", np.array([object()], dtype=object), allow_pickle=True)
    with pytest.raises(RuntimeError, match="refusing to load"):
        load_checkpoint(str(out), "cpu")
    monkeypatch.setenv("SQUISH_ALLOW_UNSAFE", "1")
    load_checkpoint(str(out), "cpu")


def test_local_model_discovery(tmp_path):
    from squish_b200.io.convert import compress
    from squish_b200.serving.model_scanner import LocalModelScanner

    sq = tmp_path / "squish"
    compress(None, str(sq / "tiny-llama-8b"), random_preset="tiny-llama", device="cpu", log=lambda *_: None)
    hf = tmp_path / "hf" / "models--Qwen--Qwen2.5-7B" / "snapshots" / "abc"
    hf.mkdir(parents=True)
    (hf / "config.json").write_text(json.dumps({"model_type": "qwen2"}))
    from safetensors.torch import save_file

    save_file({"a": torch.zeros(2)}, str(hf / "model.safetensors"))
    ol = tmp_path / "ollama"
    (ol / "manifests" / "registry" / "library" / "llama3").mkdir(parents=True)
    (ol / "blobs").mkdir()
    (ol / "blobs" / "sha256-ab").write_bytes(b"GGUF" + bytes(8))
    (ol / "manifests" / "registry" / "library" / "llama3" / "8b").write_text(json.dumps(
        {"layers": [{"mediaType": "application/vnd.ollama.image.model", "digest": "sha256:ab"}]}))
    ms = LocalModelScanner(squish_models=sq, hf_cache=tmp_path / "hf", ollama_dir=ol).find_all()
    by = {m.source: m for m in ms}
    assert by["squish"].format == "npy-dir" and by["squish"].params == "8B"
    assert by["hf-cache"].name == "Qwen/Qwen2.5-7B" and by["hf-cache"].family == "qwen2.5"
    assert by["ollama"].name == "llama3:8b" and by["ollama"].format == "gguf"


def test_startup_report_and_scan_cli(tmp_path, capsys):
    from squish_b200.cli import main
    from squish_b200.utils.startup import StartupPhase, StartupTimer, report

    report().clear()
    with StartupTimer(StartupPhase.CONFIG, "unit"):
        pass
    d = report().to_dict()
    assert d["phases"][0]["phase"] == "config" and d["phases"][0]["label"] == "unit"
    np.save(tmp_path / "a.npy", np.zeros(3))
    assert main(["scan", str(tmp_path)]) == 0
    assert json.loads(capsys.readouterr().out)["status"] == "clean"
