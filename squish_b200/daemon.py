"""``squishd``: a Unix-domain-socket daemon that keeps models resident between CLI calls.

Wire protocol (the reference's, squish/daemon/squishd.py:55-150): each message is a
4-byte big-endian length followed by that many bytes of UTF-8 JSON, at most 8 MiB. A
request with ``_cmd`` is a control command (``ping``, ``status``, ``reload``, ``stop``);
anything else is an inference request ``{model, messages | prompt, max_tokens,
temperature, top_p}`` answered with ``{text, tokens, tok_s, finish}`` or ``{error}``.
Up to ``SQUISH_MAX_MODELS`` (default 2) engines stay loaded, least recently used evicted.
The socket path is ``SQUISH_SOCK`` (default ``/tmp/squish.sock``).
"""
from __future__ import annotations

import json
import logging
import os
import socket
import struct
import threading
import time
from collections import OrderedDict
from typing import Any, Callable

log = logging.getLogger("squish_b200.daemon")

MAX_FRAME = 8 * 1024 * 1024


def sock_path() -> str:
    return os.environ.get("SQUISH_SOCK", "/tmp/squish.sock")


def max_models() -> int:
    return int(os.environ.get("SQUISH_MAX_MODELS", "2"))


def send_frame(sock: socket.socket, obj: dict) -> None:
    data = json.dumps(obj).encode()
    if len(data) > MAX_FRAME:
        raise ValueError(f"frame of {len(data)} bytes exceeds {MAX_FRAME}")
    sock.sendall(struct.pack(">I", len(data)) + data)


def _recv_exact(sock: socket.socket, n: int) -> bytes | None:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            return None
        buf += chunk
    return bytes(buf)


def recv_frame(sock: socket.socket) -> dict | None:
    head = _recv_exact(sock, 4)
    if head is None:
        return None
    (n,) = struct.unpack(">I", head)
    if n > MAX_FRAME:
        raise ValueError(f"frame of {n} bytes exceeds {MAX_FRAME}")
    body = _recv_exact(sock, n)
    return None if body is None else json.loads(body.decode())


def request(obj: dict, path: str | None = None, timeout: float = 600.0) -> dict:
    with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
        s.settimeout(timeout)
        s.connect(path or sock_path())
        send_frame(s, obj)
        resp = recv_frame(s)
    if resp is None:
        raise ConnectionError("daemon closed the connection")
    return resp


def is_running(path: str | None = None) -> bool:
    try:
        return request({"_cmd": "ping"}, path, timeout=2.0).get("status") == "ok"
    except OSError:
        return False


class _Model:
    def __init__(self, key: str, loaded):
        self.key = key
        self.loaded = loaded
        self.n_requests = 0
        self.loaded_at = time.time()
        self.last_used = self.loaded_at
        self.lock = threading.Lock()


class Daemon:
    """Serves requests on a UDS; ``loader(model) -> api.Loaded`` builds an engine."""

    def __init__(self, path: str | None = None, default_model: str | None = None,
                 loader: Callable[[str], Any] | None = None, capacity: int | None = None):
        self.path = path or sock_path()
        self.default_model = default_model
        self.capacity = capacity or max_models()
        self._loader = loader or self._default_loader
        self._models: OrderedDict[str, _Model] = OrderedDict()
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._srv: socket.socket | None = None
        self._thread: threading.Thread | None = None

    @staticmethod
    def _default_loader(model: str):
        from .api import load_engine

        return load_engine(model)

    # ------------------------------------------------------------------ lifecycle
    def start(self) -> "Daemon":
        if os.path.exists(self.path):
            if is_running(self.path):
                raise RuntimeError(f"a daemon is already listening on {self.path}")
            os.unlink(self.path)
        self._srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self._srv.bind(self.path)
        os.chmod(self.path, 0o600)
        self._srv.listen(16)
        self._srv.settimeout(0.2)
        self._thread = threading.Thread(target=self._accept_loop, name="squishd", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5.0)
        if self._srv is not None:
            self._srv.close()
        if os.path.exists(self.path):
            os.unlink(self.path)

    def serve_forever(self) -> None:
        self.start()
        try:
            while not self._stop.is_set():
                time.sleep(0.5)
        finally:
            self.stop()

    def _accept_loop(self) -> None:
        while not self._stop.is_set():
            try:
                conn, _ = self._srv.accept()
            except socket.timeout:
                continue
            except OSError:
                break
            threading.Thread(target=self._handle, args=(conn,), daemon=True).start()

    def _handle(self, conn: socket.socket) -> None:
        with conn:
            try:
                req = recv_frame(conn)
                if req is None:
                    return
                send_frame(conn, self.dispatch(req))
            except (OSError, ValueError) as exc:
                try:
                    send_frame(conn, {"error": str(exc)})
                except OSError:
                    pass

    # ------------------------------------------------------------------ commands
    def dispatch(self, req: dict) -> dict:
        cmd = req.get("_cmd")
        if cmd == "ping":
            with self._lock:
                return {"status": "ok", "models": list(self._models), "pid": os.getpid()}
        if cmd == "status":
            with self._lock:
                info = {k: {"n_requests": m.n_requests, "loaded_at": m.loaded_at, "last_used": m.last_used}
                        for k, m in self._models.items()}
            return {"status": "ok", "pid": os.getpid(), "models": info}
        if cmd == "reload":
            key = req.get("model") or self.default_model
            with self._lock:
                self._models.pop(key, None)
            try:
                self._get(key)
            except (OSError, ValueError, RuntimeError, KeyError) as exc:
                return {"error": str(exc)}
            return {"status": "ok", "reloaded": key}
        if cmd == "stop":
            self._stop.set()
            return {"status": "ok", "stopping": True}
        if cmd is not None:
            return {"error": f"unknown command {cmd!r}"}
        return self._infer(req)

    def _get(self, key: str) -> _Model:
        with self._lock:
            m = self._models.get(key)
            if m is not None:
                self._models.move_to_end(key)
                return m
        loaded = self._loader(key)
        with self._lock:
            m = self._models[key] = _Model(key, loaded)
            while len(self._models) > self.capacity:
                old, _ = self._models.popitem(last=False)
                log.info("evicted %s", old)
        return m

    def _infer(self, req: dict) -> dict:
        from .engine.sampling import SamplingParams
        from .serving.chat_template import apply_chat_template

        key = req.get("model") or self.default_model
        if not key:
            return {"error": "no model given and no default model"}
        try:
            m = self._get(key)
        except (OSError, ValueError, RuntimeError, KeyError) as exc:
            return {"error": f"model not available: {key}: {exc}"}
        tok = m.loaded.tokenizer
        if "messages" in req:
            text = apply_chat_template(req["messages"], tok, arch=getattr(m.loaded.engine.cfg, "arch", "qwen2"))
        else:
            text = str(req.get("prompt", ""))
        try:
            params = SamplingParams(max_tokens=int(req.get("max_tokens", 512)),
                                    temperature=float(req.get("temperature", 0.7)),
                                    top_p=float(req.get("top_p", 0.9)),
                                    stop_token_ids=[m.loaded.engine.cfg.eos_token_id]).validate()
        except (TypeError, ValueError) as exc:
            return {"error": str(exc)}
        t0 = time.perf_counter()
        with m.lock:  # the engine is single-threaded; requests to one model run in turn
            eng = m.loaded.engine
            rid = eng.add_request(tok.encode(text), params)
            out: list[int] = []
            reason = None
            while eng.has_unfinished():
                for o in eng.step():
                    if o.rid == rid:
                        out.extend(o.new_tokens)
                        if o.finished:
                            reason = o.finish_reason
        dt = time.perf_counter() - t0
        with self._lock:
            m.n_requests += 1
            m.last_used = time.time()
        return {"text": tok.decode(out), "tokens": len(out), "tok_s": round(len(out) / dt, 2) if dt > 0 else 0.0,
                "finish": reason or "stop"}
