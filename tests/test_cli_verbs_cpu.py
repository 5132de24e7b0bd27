"""The client and local CLI verbs (chat, info, search, rm, ps, logs, trace, quality, route,
export, eval, push) against a live HTTP server over the CPU engine."""
import io
import json
import socket
import sys
import threading
import time

import pytest

from squish_b200.cli import main


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def server():
    import uvicorn

    from squish_b200.engine.engine import EngineConfig, LLMEngine
    from squish_b200.models.config import get_preset
    from squish_b200.models.weights import random_checkpoint
    from squish_b200.serving.async_engine import AsyncEngine
    from squish_b200.serving.server import ServerState, create_app
    from squish_b200.serving.tokenizer import ByteTokenizer

    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0), "cpu",
                                    EngineConfig(max_num_seqs=4, max_model_len=512, num_pages=128))
    aeng = AsyncEngine(eng, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id), model_name="tiny").start()
    port = _port()
    srv = uvicorn.Server(uvicorn.Config(create_app(ServerState(aeng, "tiny", api_key=None, arch="llama")),
                                        host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    for _ in range(200):
        if srv.started:
            break
        time.sleep(0.05)
    yield port
    srv.should_exit = True
    th.join(timeout=10)
    aeng.stop()


def _run(argv, capsys, stdin=None, monkeypatch=None):
    if stdin is not None:
        monkeypatch.setattr(sys, "stdin", io.StringIO(stdin))
    rc = main(argv)
    out = capsys.readouterr()
    return rc, out.out, out.err


def test_client_verbs(server, capsys, monkeypatch, tmp_path):
    p = ["--port", str(server)]
    rc, out, _ = _run(["ps"] + p, capsys)
    assert rc == 0 and json.loads(out.splitlines()[0])["name"] == "tiny"
    rc, out, _ = _run(["quality"] + p, capsys)
    assert rc == 0 and "total_requests" in json.loads(out)
    rc, out, _ = _run(["route", "write", "a", "python", "function"] + p, capsys)
    assert rc == 0 and isinstance(json.loads(out), dict)
    rc, out, _ = _run(["trace", "obs"] + p, capsys)
    assert rc == 0 and isinstance(json.loads(out), dict)
    rc, out, _ = _run(["trace"] + p, capsys)
    assert rc == 0
    chrome = tmp_path / "t.json"
    rc, out, _ = _run(["trace", "--chrome", str(chrome)] + p, capsys)
    assert rc == 0 and chrome.exists() and json.loads(chrome.read_text()) is not None
    rc, out, _ = _run(["trace", "reset"] + p, capsys)
    assert rc == 0
    rc, out, _ = _run(["chat", "--url", f"http://127.0.0.1:{server}", "--max-tokens", "4", "--temperature", "0"],
                      capsys, stdin="hello\nagain\n\n", monkeypatch=monkeypatch)
    assert rc == 0 and len(out.splitlines()) == 2
    rc, _, err = _run(["ps", "--port", str(_port())], capsys)
    assert rc == 1 and "no squish server" in err


def test_local_verbs(capsys, monkeypatch, tmp_path):
    monkeypatch.setenv("SQUISH_HOME", str(tmp_path))
    rc, out, _ = _run(["info", "tiny-llama"], capsys)
    info = json.loads(out)
    assert rc == 0 and info["layers"] == 4 and info["arch"] == "llama"
    rc, out, _ = _run(["search", "qwen"], capsys)
    assert rc == 0 and "qwen2.5-7b" in out
    assert _run(["search", "no-such-model-xyz"], capsys)[0] == 1
    # pull writes a random-init checkpoint under $SQUISH_HOME/models; info, export, rm on it
    rc, out, _ = _run(["pull", "tiny-llama", "--device", "cpu"], capsys)
    assert rc == 0
    mdir = tmp_path / "models" / "tiny-llama"
    assert mdir.exists()
    rc, out, _ = _run(["info", str(mdir)], capsys)
    assert rc == 0 and json.loads(out)["kind"] == "checkpoint"
    dest = tmp_path / "tiny.squizd"
    rc, out, _ = _run(["export", str(mdir), str(dest)], capsys)
    assert rc == 0 and dest.exists()
    outside = tmp_path.parent / f"keep-{tmp_path.name}"
    outside.mkdir()
    assert _run(["rm", str(outside), "--yes"], capsys)[0] == 2 and outside.exists()
    outside.rmdir()
    rc, out, _ = _run(["rm", "tiny-llama", "--yes"], capsys)
    assert rc == 0 and not mdir.exists()
    assert _run(["push", "x"], capsys)[0] == 2
    # the server log that `squish serve` appends to
    logf = tmp_path / "logs" / "server.log"
    logf.parent.mkdir(parents=True)
    logf.write_text("".join(f"line {i}\n" for i in range(100)))
    rc, out, _ = _run(["logs", "-n", "3"], capsys)
    assert rc == 0 and out.splitlines() == ["line 97", "line 98", "line 99"]


def test_eval_perplexity_of_random_tokens(capsys):
    rc, out, _ = _run(["eval", "tiny-llama", "--max-tokens", "96", "--window", "48"], capsys)
    d = json.loads(out)
    assert rc == 0 and d["tokens"] == 95
    # random weights give a near-uniform next-token distribution over the 32000-token vocabulary
    assert 0.5 * 32000 < d["perplexity"] < 2.0 * 32000
