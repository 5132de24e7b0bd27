"""Local model discovery and a static safety scan of model files before loading.

The reference's scanner (squish/serving/local_model_scanner.py) lists models found under the
squish models directory, Ollama and LM Studio, and ``scan_before_load`` (:317-440) inspects
files without executing them: pickle files for code-importing opcodes, GGUF magic, and the
safetensors header length. Here the pickle check walks the opcode stream with ``pickletools``
(a parser, nothing is unpickled), so a byte that merely equals an opcode value elsewhere in the
file is not a finding; ``.npy`` files holding Python objects (which np.load can only read by
unpickling) are flagged too, and the safetensors JSON header must parse.
"""
from __future__ import annotations

import io
import json
import os
import pickletools
import re
import struct
import zipfile
from dataclasses import dataclass, field
from pathlib import Path

_PICKLE_EXT = {".bin", ".pt", ".pth", ".pkl", ".pickle", ".ckpt"}
_CODE_OPS = {"GLOBAL", "STACK_GLOBAL", "REDUCE", "INST", "OBJ", "NEWOBJ", "NEWOBJ_EX", "BUILD"}
# the GLOBALs torch's own checkpoints need to rebuild tensors (no other code runs)
_TORCH_SAFE = re.compile(r"^(torch\._utils _rebuild_\w+|torch \w+Storage|torch \w+|collections OrderedDict|"
                         r"torch\._tensor _rebuild_from_type_v2|builtins (set|frozenset|bytearray|slice))$")


@dataclass
class ScanResult:
    status: str                      # "clean" | "unsafe" | "error"
    findings: list[str] = field(default_factory=list)
    scanned: int = 0


def _pickle_findings(name: str, data: bytes) -> list[str]:
    out, globals_seen = [], []
    try:
        prev_strings: list[str] = []
        for op, arg, pos in pickletools.genops(io.BytesIO(data)):
            if op.name in ("SHORT_BINUNICODE", "BINUNICODE", "UNICODE", "BINUNICODE8"):
                prev_strings = (prev_strings + [str(arg)])[-2:]
            if op.name == "GLOBAL":
                globals_seen.append(str(arg).replace("\n", " "))
            elif op.name == "STACK_GLOBAL":
                globals_seen.append(" ".join(prev_strings))
            elif op.name == "STOP":
                break
    except Exception as exc:  # noqa: BLE001 - a malformed stream is itself a finding
        return [f"[UNSAFE] {name}: unparseable pickle stream ({type(exc).__name__})"]
    bad = [g for g in globals_seen if not _TORCH_SAFE.match(g)]
    if bad:
        out.append(f"[UNSAFE] {name}: pickle imports {sorted(set(bad))[:5]}")
    return out


def _scan_pickle(path: Path) -> list[str]:
    try:
        if zipfile.is_zipfile(path):  # torch.save zip container: scan every data.pkl
            with zipfile.ZipFile(path) as z:
                return [f for n in z.namelist() if n.endswith(".pkl") for f in _pickle_findings(
                    f"{path.name}:{n}", z.read(n))]
        return _pickle_findings(path.name, path.read_bytes())
    except OSError as exc:
        return [f"[READ ERROR] {path.name}: {exc}"]


def _scan_npy(path: Path) -> list[str]:
    import numpy as np

    try:
        with open(path, "rb") as f:
            version = np.lib.format.read_magic(f)
            read = {1: np.lib.format.read_array_header_1_0, 2: np.lib.format.read_array_header_2_0}.get(version[0])
            if read is None:
                return [f"[UNSAFE] {path.name}: unsupported .npy version {version}"]
            shape, fortran, dtype = read(f)  # the header only
    except Exception as exc:  # noqa: BLE001
        return [f"[UNSAFE] {path.name}: invalid .npy header ({type(exc).__name__})"]
    if dtype.hasobject:
        return [f"[UNSAFE] {path.name}: .npy holds Python objects (loading would unpickle)"]
    return []


def _scan_gguf(path: Path) -> list[str]:
    try:
        with open(path, "rb") as f:
            magic = f.read(4)
    except OSError as exc:
        return [f"[READ ERROR] {path.name}: {exc}"]
    return [] if magic == b"GGUF" else [f"[UNSAFE] {path.name}: invalid GGUF magic {magic!r}"]


def _scan_safetensors(path: Path) -> list[str]:
    try:
        size = path.stat().st_size
        with open(path, "rb") as f:
            raw = f.read(8)
            if len(raw) < 8:
                return [f"[UNSAFE] {path.name}: truncated safetensors header"]
            (hlen,) = struct.unpack("<Q", raw)
            if hlen == 0 or hlen + 8 > size or hlen > 100 * 2**20:
                return [f"[UNSAFE] {path.name}: header length {hlen} is implausible for a {size}-byte file"]
            hdr = json.loads(f.read(hlen))
    except (OSError, ValueError) as exc:
        return [f"[UNSAFE] {path.name}: unreadable safetensors header ({type(exc).__name__})"]
    end = 8 + hlen
    for k, v in hdr.items():
        if k == "__metadata__":
            continue
        off = v.get("data_offsets", [0, 0]) if isinstance(v, dict) else [0, 0]
        if not (0 <= off[0] <= off[1] and end + off[1] <= size):
            return [f"[UNSAFE] {path.name}: tensor {k!r} lies outside the file"]
    return []


def scan_before_load(path: str | Path) -> ScanResult:
    """Inspect every model file under ``path`` (a directory or one file) without executing it."""
    p = Path(path)
    if not p.exists():
        return ScanResult("error", [f"not found: {p}"])
    files = [p] if p.is_file() else sorted(f for f in p.rglob("*") if f.is_file())
    findings, n = [], 0
    for f in files:
        suf = f.suffix.lower()
        if suf in _PICKLE_EXT:
            res = _scan_pickle(f)
        elif suf == ".npy":
            res = _scan_npy(f)
        elif suf == ".gguf":
            res = _scan_gguf(f)
        elif suf == ".safetensors":
            res = _scan_safetensors(f)
        else:
            continue
        n += 1
        findings += res
    return ScanResult("unsafe" if any(x.startswith("[UNSAFE]") for x in findings) else
                      ("error" if findings else "clean"), findings, n)


# ------------------------------------------------------------------------------ discovery
@dataclass
class LocalModel:
    name: str
    path: str
    source: str        # "squish" | "hf-cache" | "ollama" | "extra"
    format: str
    bytes: int
    family: str = ""
    params: str = ""


def _guess_family(name: str) -> str:
    n = name.lower()
    for fam in ("qwen3", "qwen2.5", "qwen2", "qwen", "llama", "mistral", "mixtral", "gemma", "phi", "deepseek"):
        if fam in n:
            return fam
    return ""


def _guess_params(name: str) -> str:
    m = re.search(r"(\d+(?:\.\d+)?)\s*[bB](?![a-z])", name)
    return f"{m.group(1)}B" if m else ""


def _size(p: Path) -> int:
    if p.is_file():
        return p.stat().st_size
    return sum(f.stat().st_size for f in p.rglob("*") if f.is_file())


class LocalModelScanner:
    def __init__(self, squish_models: Path | None = None, extra_dirs: list[Path] | None = None,
                 hf_cache: Path | None = None, ollama_dir: Path | None = None):
        from .. import config as ucfg

        self.squish_models = squish_models or ucfg.squish_home() / "models"
        self.extra_dirs = list(extra_dirs or [])
        self.hf_cache = hf_cache or Path(os.environ.get("HF_HUB_CACHE", Path.home() / ".cache/huggingface/hub"))
        self.ollama_dir = ollama_dir or Path(os.environ.get("OLLAMA_MODELS", Path.home() / ".ollama/models"))

    def _dir_models(self, root: Path, source: str) -> list[LocalModel]:
        from ..io.npy_dir import detect_format

        out = []
        if not root.is_dir():
            return out
        for p in sorted(root.iterdir()):
            if p.name.startswith("."):
                continue
            try:
                fmt = detect_format(p)
            except (ValueError, OSError):
                continue
            out.append(LocalModel(p.name, str(p), source, fmt, _size(p), _guess_family(p.name), _guess_params(p.name)))
        return out

    def scan_squish(self) -> list[LocalModel]:
        return self._dir_models(self.squish_models, "squish") + \
            [m for d in self.extra_dirs for m in self._dir_models(d, "extra")]

    def scan_hf_cache(self) -> list[LocalModel]:
        from ..io.npy_dir import detect_format

        out = []
        if not self.hf_cache.is_dir():
            return out
        for repo in sorted(self.hf_cache.glob("models--*")):
            snaps = sorted((repo / "snapshots").glob("*"), key=lambda q: q.stat().st_mtime)
            if not snaps:
                continue
            try:
                fmt = detect_format(snaps[-1])
            except (ValueError, OSError):
                continue
            name = repo.name[len("models--"):].replace("--", "/")
            out.append(LocalModel(name, str(snaps[-1]), "hf-cache", fmt, _size(repo / "blobs") if
                                  (repo / "blobs").is_dir() else _size(snaps[-1]), _guess_family(name),
                                  _guess_params(name)))
        return out

    def scan_ollama(self) -> list[LocalModel]:
        """Ollama manifests name GGUF blobs; the blob (a GGUF file) is the loadable path."""
        out = []
        man = self.ollama_dir / "manifests"
        if not man.is_dir():
            return out
        for f in sorted(man.rglob("*")):
            if not f.is_file():
                continue
            try:
                layers = json.loads(f.read_text()).get("layers", [])
            except (OSError, ValueError):
                continue
            for layer in layers:
                if layer.get("mediaType", "").endswith(".model"):
                    blob = self.ollama_dir / "blobs" / layer.get("digest", "").replace(":", "-")
                    if blob.exists():
                        name = f"{f.parent.name}:{f.name}"
                        out.append(LocalModel(name, str(blob), "ollama", "gguf", blob.stat().st_size,
                                              _guess_family(name), _guess_params(name)))
        return out

    def find_all(self) -> list[LocalModel]:
        seen, out = set(), []
        for m in self.scan_squish() + self.scan_hf_cache() + self.scan_ollama():
            if m.path not in seen:
                seen.add(m.path)
                out.append(m)
        return out
