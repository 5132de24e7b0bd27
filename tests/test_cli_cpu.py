"""CLI, user config, UDS daemon protocol, offline LLM API and the serving load generator (CPU).

Mirrors the reference's tests/test_config.py, tests/test_squishd.py and the CLI smoke tests:
config dot-keys and env overrides, 4-byte big-endian length-prefixed JSON frames, LRU of
loaded models, and the verbs that need no GPU.
"""
import json
import socket
import struct
import threading

import pytest

from squish_b200 import cli, config as ucfg, daemon
from squish_b200.engine.engine import EngineConfig


@pytest.fixture()
def home(tmp_path, monkeypatch):
    monkeypatch.setenv("SQUISH_HOME", str(tmp_path / "home"))
    monkeypatch.delenv("SQUISH_CONFIG_DIR", raising=False)
    return tmp_path / "home"


def test_config_defaults_set_get_reset(home, monkeypatch):
    assert ucfg.get("server.port") == 11435 and ucfg.get("server.host") == "127.0.0.1"
    assert ucfg.get("server.api_key") == "squish"
    ucfg.set_value("server.port", "8080")
    ucfg.set_value("engine.cuda_graphs", "false")
    assert ucfg.get("server.port") == 8080 and ucfg.get("engine.cuda_graphs") is False
    assert json.loads((home / "config.json").read_text())["server"]["port"] == 8080
    ucfg.reset()
    assert ucfg.get("server.port") == 11435
    monkeypatch.setenv("SQUISH_CONFIG_DIR", str(home / "elsewhere"))
    assert ucfg.config_path() == home / "elsewhere" / "config.json"


def test_cli_config_catalog_version(home, capsys):
    assert cli.main(["config", "set", "model.default", "tiny-llama"]) == 0
    assert cli.main(["config", "get", "model.default"]) == 0
    assert capsys.readouterr().out.strip().splitlines()[-1] == '"tiny-llama"'
    assert cli.main(["catalog"]) == 0
    d = json.loads(capsys.readouterr().out)
    names = [r["name"] for r in d["presets"]]
    assert "qwen2.5-7b" in names and "llama-3-70b" in names
    assert "qwen2.5:7b" in [e["id"] for e in d["catalog"]]
    assert cli.main(["version"]) == 0


def test_cli_pull_offline_and_models(home, capsys):
    assert cli.main(["pull", "some-org/unknown-model"]) == 2
    assert cli.main(["pull", "tiny-llama", "--device", "cpu"]) == 0
    capsys.readouterr()
    assert cli.main(["models"]) == 0
    local = json.loads(capsys.readouterr().out)["local"]
    assert local[0]["name"] == "tiny-llama" and local[0]["format"] == "npy-dir"


def test_cli_run_one_shot_on_cpu(home, capsys):
    rc = cli.main(["run", "tiny-llama", "hello", "--device", "cpu", "--max-tokens", "4", "--max-model-len", "256",
                   "--max-num-seqs", "2", "--no-cuda-graphs"])
    assert rc == 0


def test_cli_doctor_reports(capsys):
    rep = cli.doctor_report()
    assert rep["extension"] == "loaded" and "torch" in rep


def test_frame_codec_and_limits():
    a, b = socket.socketpair()
    b.settimeout(5)
    daemon.send_frame(a, {"x": 1, "s": "é"})
    body = json.dumps({"x": 1, "s": "é"}).encode()
    assert b.recv(4) == struct.pack(">I", len(body))
    assert json.loads(daemon._recv_exact(b, len(body))) == {"x": 1, "s": "é"}
    a.sendall(struct.pack(">I", 3) + b"[1]")
    assert daemon.recv_frame(b) == [1]
    a.sendall(struct.pack(">I", daemon.MAX_FRAME + 1))
    with pytest.raises(ValueError):
        daemon.recv_frame(b)
    a.close()
    assert daemon.recv_frame(b) is None
    b.close()


class _FakeLoaded:
    def __init__(self, key):
        from squish_b200.engine.engine import LLMEngine
        from squish_b200.models.config import get_preset
        from squish_b200.models.weights import random_checkpoint
        from squish_b200.serving.tokenizer import ByteTokenizer

        cfg, q = get_preset("tiny-llama")
        self.engine = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0), "cpu",
                                                EngineConfig(max_num_seqs=4, max_model_len=256, num_pages=64))
        self.tokenizer = ByteTokenizer(cfg.vocab_size, cfg.eos_token_id)
        self.key = key


def test_daemon_protocol_lru_and_inference(tmp_path):
    loads = []

    def loader(key):
        loads.append(key)
        return _FakeLoaded(key)

    path = str(tmp_path / "s.sock")
    d = daemon.Daemon(path, default_model="a", loader=loader, capacity=2).start()
    try:
        assert daemon.is_running(path)
        r = daemon.request({"prompt": "hi", "max_tokens": 3, "temperature": 0}, path)
        assert r["tokens"] >= 1 and "text" in r and r["finish"] in ("length", "stop")
        daemon.request({"model": "b", "prompt": "x", "max_tokens": 1}, path)
        daemon.request({"model": "a", "prompt": "y", "max_tokens": 1}, path)  # a becomes most recent
        daemon.request({"model": "c", "prompt": "z", "max_tokens": 1}, path)  # evicts b
        st = daemon.request({"_cmd": "status"}, path)
        assert sorted(st["models"]) == ["a", "c"] and st["models"]["a"]["n_requests"] == 2
        assert loads == ["a", "b", "c"]
        assert daemon.request({"_cmd": "reload", "model": "a"}, path)["reloaded"] == "a"
        assert loads[-1] == "a"
        assert "error" in daemon.request({"_cmd": "nope"}, path)
        # concurrent clients on the same model are serialised, not corrupted
        res = []
        ts = [threading.Thread(target=lambda: res.append(daemon.request({"prompt": "q", "max_tokens": 2}, path)))
              for _ in range(3)]
        [t.start() for t in ts]
        [t.join() for t in ts]
        assert all(r["tokens"] == 2 or r["finish"] == "stop" for r in res) and len(res) == 3
    finally:
        d.stop()
    assert not daemon.is_running(path)


def test_llm_api_and_loadgen_cpu():
    from squish_b200.api import LLM
    from squish_b200.engine.sampling import SamplingParams
    from squish_b200.utils.loadgen import run_load

    llm = LLM("tiny-llama", "cpu", ecfg=EngineConfig(max_num_seqs=4, max_model_len=256, num_pages=128,
                                                      cuda_graphs=False))
    outs = llm.generate([[1, 2, 3], [4, 5]], SamplingParams(max_tokens=3, ignore_eos=True))
    assert [len(o["token_ids"]) for o in outs] == [3, 3] and outs[0]["finish_reason"] == "length"
    r = run_load(llm.engine, num_requests=5, concurrency=2, prompt_min=4, prompt_max=12, max_tokens=3)
    assert r["requests"] == 5 and r["output_tokens"] == 15 and r["ttft_ms_p50"] > 0


def test_nvlink_topology_from_nvml_queries():
    """The doctor's NVLink report from (read-only) NVML queries, against a stand-in NVML of two
    GPUs with 18 links up and NVLink P2P between them."""
    class FakeNVML:
        NVML_NVLINK_MAX_LINKS = 18
        NVML_FEATURE_ENABLED = 1
        NVML_P2P_CAPS_INDEX_NVLINK = 3
        NVML_P2P_STATUS_OK = 0
        calls = []

        def nvmlInit(self): self.calls.append("init")
        def nvmlShutdown(self): self.calls.append("shutdown")
        def nvmlDeviceGetCount(self): return 2
        def nvmlDeviceGetHandleByIndex(self, i): return f"h{i}"
        def nvmlDeviceGetNvLinkState(self, h, ln): return 1
        def nvmlDeviceGetP2PStatus(self, a, b, idx):
            assert idx == 3
            return 0

    f = FakeNVML()
    topo = cli.nvlink_topology(f)
    assert topo == [{"index": 0, "nvlinks_up": 18, "nvlink_p2p": {1: True}},
                    {"index": 1, "nvlinks_up": 18, "nvlink_p2p": {0: True}}]
    assert f.calls == ["init", "shutdown"]
    # no driver: nothing to report
    class NoDriver(FakeNVML):
        def nvmlInit(self): raise RuntimeError("NVML Shared Library Not Found")
    assert cli.nvlink_topology(NoDriver()) is None
