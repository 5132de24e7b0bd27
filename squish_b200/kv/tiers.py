"""Host-RAM and disk tiers behind the device prefix cache.

When the block manager reuses a cached page (a full block of some earlier sequence, ref 0)
for new data, the page's contents are first copied to a host LRU keyed by the block's
chained hash; when the host tier is over its byte budget, its oldest blocks spill to a
disk directory as ``<hash>.npz`` files. ``match_prefix`` that runs out of device hits
continues with the tiers: every further block found there is copied into a fresh device
page and published again, so a long shared prefix survives device-pool pressure and
process restarts.

The disk directory carries ``manifest.json`` (page size, model key, KV format, group,
layers, heads, head dim); a directory written for a different model or cache layout is
ignored at boot. Page contents are the device bytes as they are (quantized codes and
scales), so restoring is bit-exact.

This is the counterpart of the reference's BlockKVCache hot RAM + cold disk tiers and its
manifest check (squish/kv/block_kv_cache.py:1-60, 118-140, 584-636), on device pages.
"""
from __future__ import annotations

import json
import os
from collections import OrderedDict
from pathlib import Path

import numpy as np
import torch


class PageIO:
    """Reads / writes one device page of every layer (all tensors of the page)."""

    def __init__(self, runner):
        self.runner = runner

    def _tensors(self) -> list[torch.Tensor]:
        r = self.runner
        if hasattr(r, "pools"):  # CudaRunner: [num_pages, Hkv, page, bytes] per layer and kind
            return [t for layer in r.pools.layers for t in layer]
        return [r.k, r.v]  # CPU runner: dense [L, P, Hkv, page, D]

    def read(self, page: int) -> list[np.ndarray]:
        r = self.runner
        if hasattr(r, "pools"):
            return [t[page].cpu().numpy().copy() for t in self._tensors()]
        return [r.k[:, page].numpy().copy(), r.v[:, page].numpy().copy()]

    def write(self, page: int, arrays: list[np.ndarray]) -> None:
        r = self.runner
        if hasattr(r, "pools"):
            for t, a in zip(self._tensors(), arrays):
                t[page].copy_(torch.from_numpy(a), non_blocking=False)
        else:
            r.k[:, page] = torch.from_numpy(arrays[0])
            r.v[:, page] = torch.from_numpy(arrays[1])


class KVTierStore:
    def __init__(self, io: PageIO, layout: dict, host_bytes: int = 2 << 30, disk_dir: str | None = None,
                 disk_bytes: int = 8 << 30):
        self.io = io
        self.layout = dict(layout, format_version=1)
        self.host_bytes, self.disk_bytes = host_bytes, disk_bytes
        self.host: OrderedDict[bytes, list[np.ndarray]] = OrderedDict()
        self.host_used = 0
        self.disk_dir = Path(disk_dir) if disk_dir else None
        self.disk: OrderedDict[bytes, int] = OrderedDict()  # hash -> file bytes, oldest first
        self.stats = {"offloaded": 0, "restored_host": 0, "restored_disk": 0, "spilled": 0, "dropped": 0}
        if self.disk_dir is not None:
            self._open_disk()

    # ------------------------------------------------------------------ disk
    def _open_disk(self) -> None:
        self.disk_dir.mkdir(parents=True, exist_ok=True)
        man = self.disk_dir / "manifest.json"
        if man.exists():
            try:
                old = json.loads(man.read_text())
            except (OSError, ValueError):
                old = None
            if old != self.layout:
                # another model or cache layout: ignore (and replace) what is there
                for f in self.disk_dir.glob("*.npz"):
                    f.unlink()
        man.write_text(json.dumps(self.layout, indent=2, sort_keys=True))
        files = sorted(self.disk_dir.glob("*.npz"), key=lambda f: f.stat().st_mtime)
        for f in files:
            self.disk[bytes.fromhex(f.stem)] = f.stat().st_size

    def _disk_path(self, h: bytes) -> Path:
        return self.disk_dir / f"{h.hex()}.npz"

    def _spill(self, h: bytes, arrays: list[np.ndarray]) -> None:
        if self.disk_dir is None:
            self.stats["dropped"] += 1
            return
        path = self._disk_path(h)
        tmp = path.with_suffix(".tmp.npz")
        np.savez(tmp, *arrays)
        os.replace(tmp, path)
        self.disk[h] = path.stat().st_size
        self.stats["spilled"] += 1
        while sum(self.disk.values()) > self.disk_bytes and self.disk:
            old, _ = self.disk.popitem(last=False)
            try:
                self._disk_path(old).unlink()
            except OSError:
                pass

    # ------------------------------------------------------------------ tiers
    def offload(self, h: bytes, page: int) -> None:
        """Keep a copy of device page ``page`` (block hash ``h``) before it is reused."""
        if h in self.host or h in self.disk:
            return
        arrays = self.io.read(page)
        self.host[h] = arrays
        self.host_used += sum(a.nbytes for a in arrays)
        self.stats["offloaded"] += 1
        while self.host_used > self.host_bytes and self.host:
            old, arr = self.host.popitem(last=False)
            self.host_used -= sum(a.nbytes for a in arr)
            self._spill(old, arr)

    def has(self, h: bytes) -> bool:
        return h in self.host or h in self.disk

    def restore(self, h: bytes, page: int) -> bool:
        """Copy block ``h`` into device page ``page``; False if no tier has it."""
        if h in self.host:
            self.host.move_to_end(h)
            self.io.write(page, self.host[h])
            self.stats["restored_host"] += 1
            return True
        if h in self.disk:
            try:
                with np.load(self._disk_path(h)) as z:
                    arrays = [z[f"arr_{i}"] for i in range(len(z.files))]
            except (OSError, ValueError):
                self.disk.pop(h, None)
                return False
            self.disk.move_to_end(h)
            self.io.write(page, arrays)
            self.stats["restored_disk"] += 1
            return True
        return False

    def flush(self) -> int:
        """Write every host-tier block to disk (e.g. before shutdown); returns blocks written."""
        if self.disk_dir is None:
            return 0
        n = 0
        for h, arr in list(self.host.items()):
            if h not in self.disk:
                self._spill(h, arr)
                n += 1
        return n


def layout_of(cfg, qcfg, num_layers: int | None = None, hkv: int | None = None) -> dict:
    return {"page_size": qcfg.page_size, "model": cfg.name, "kv_dtype": qcfg.kv_dtype, "kv_group": qcfg.kv_group,
            "layers": num_layers or cfg.num_layers, "kv_heads": hkv or cfg.num_kv_heads, "head_dim": cfg.head_dim}
