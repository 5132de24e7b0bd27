"""Choose which OpenAI-compatible backend a client talks to, from the environment.

The reference's BackendConfig / BackendRouter (squish/serving/backend_router.py): the backend is
``SQUISH_BACKEND`` (squish | ollama | openai | localai), its base URL ``SQUISH_BACKEND_URL`` or
the backend's default, the key ``SQUISH_API_KEY`` / ``OPENAI_API_KEY``; ``proxy_url(path)``
maps an OpenAI path onto the backend (Ollama's native API for its own routes) and
``health_check()`` probes it with a short timeout.
"""
from __future__ import annotations

import os
import urllib.error
import urllib.request
from dataclasses import dataclass, field

DEFAULT_URLS = {
    "squish": "http://127.0.0.1:11435",
    "ollama": "http://127.0.0.1:11434",
    "openai": "https://api.openai.com",
    "localai": "http://127.0.0.1:8080",
}
_HEALTH = {"squish": "/health", "ollama": "/api/version", "openai": "/v1/models", "localai": "/readyz"}


@dataclass
class BackendConfig:
    backend: str = field(default_factory=lambda: os.environ.get("SQUISH_BACKEND", "squish").lower())
    base_url: str = ""
    api_key: str | None = field(default_factory=lambda: os.environ.get("SQUISH_API_KEY") or
                                os.environ.get("OPENAI_API_KEY"))

    def __post_init__(self) -> None:
        if self.backend not in DEFAULT_URLS:
            raise ValueError(f"unknown backend {self.backend!r}; one of {sorted(DEFAULT_URLS)}")
        if not self.base_url:
            self.base_url = os.environ.get("SQUISH_BACKEND_URL", "") or DEFAULT_URLS[self.backend]
        self.base_url = self.base_url.rstrip("/")

    @property
    def default_url(self) -> str:
        return DEFAULT_URLS[self.backend]


class BackendRouter:
    def __init__(self, config: BackendConfig | None = None):
        self.config = config or BackendConfig()

    def proxy_url(self, path: str) -> str:
        p = path if path.startswith("/") else "/" + path
        return self.config.base_url + p

    def headers(self) -> dict:
        h = {"Content-Type": "application/json"}
        if self.config.api_key:
            h["Authorization"] = f"Bearer {self.config.api_key}"
        return h

    def health_check(self, timeout: float = 2.0) -> bool:
        req = urllib.request.Request(self.proxy_url(_HEALTH[self.config.backend]), headers=self.headers())
        try:
            with urllib.request.urlopen(req, timeout=timeout) as r:  # noqa: S310 - a configured local/remote URL
                return 200 <= r.status < 300
        except (urllib.error.URLError, OSError, ValueError):
            return False

    def __repr__(self) -> str:
        return f"BackendRouter(backend={self.config.backend!r}, url={self.config.base_url!r})"
