"""Image bytes from local, immutable TAR shards by (shard, offset, length, sha256) locators.

``ImageReader.read_bytes`` validates the locator (relative path inside the source root, range
inside the recorded shard size), reads the range with ``os.pread`` on a duplicated descriptor
taken from a small LRU of open shards, and checks the payload's sha256. The duplicate is a
lease: evicting the shard's cached descriptor never closes one that a concurrent read is using.
``read`` decodes with PIL, applies the EXIF orientation, converts to RGB and, unless
``native_resolution``, centre-crops and resizes to ``image_size`` (reference
``data/images.py:25-100``).
"""

from __future__ import annotations

import hashlib
import io
import os
import threading
from collections import OrderedDict
from pathlib import Path

import numpy as np


class ImageReader:
    def __init__(self, source_root, shard_sizes, image_size=512, native_resolution=False, max_open=32,
                 max_bytes=256 << 20):
        self.root = Path(source_root).resolve()
        self.sizes = dict(shard_sizes)
        self.image_size, self.native_resolution = image_size, native_resolution
        self.max_open, self.max_bytes = max_open, max_bytes
        self._fds: OrderedDict = OrderedDict()
        self._lock = threading.Lock()
        self.counters = dict(images=0, bytes=0, reads=0)

    def _lease(self, shard):
        """A private duplicate of the shard's cached descriptor (caller closes it)."""
        with self._lock:
            fd = self._fds.get(shard)
            if fd is None:
                path = (self.root / shard).resolve()
                if not path.is_relative_to(self.root):
                    raise ValueError(f"shard escapes the source root: {shard}")
                fd = os.open(path, os.O_RDONLY)
                if os.fstat(fd).st_size != self.sizes[shard]:
                    os.close(fd)
                    raise RuntimeError(f"shard size changed: {shard}")
                self._fds[shard] = fd
            self._fds.move_to_end(shard)
            lease = os.dup(fd)
            while len(self._fds) > self.max_open:
                os.close(self._fds.popitem(last=False)[1])
            return lease

    def read_bytes(self, locator) -> bytes:
        shard = locator["shard"]
        p = Path(shard)
        if p.is_absolute() or ".." in p.parts or "://" in shard:
            raise ValueError(f"expected a relative local shard path: {shard}")
        if shard not in self.sizes:
            raise ValueError(f"unknown shard: {shard}")
        offset, length = int(locator["offset"]), int(locator["length"])
        if offset < 0 or not 0 < length <= self.max_bytes or offset + length > self.sizes[shard]:
            raise ValueError(f"invalid range {shard}:{offset}+{length}")
        fd = self._lease(shard)
        try:
            body = os.pread(fd, length, offset)
        finally:
            os.close(fd)
        if len(body) != length or hashlib.sha256(body).hexdigest() != locator["sha256"]:
            raise RuntimeError(f"image integrity failure at {shard}:{offset}")
        with self._lock:
            self.counters["bytes"] += length
            self.counters["reads"] += 1
        return body

    def read(self, locator) -> np.ndarray:
        from PIL import Image, ImageOps
        body = self.read_bytes(locator)
        with Image.open(io.BytesIO(body)) as image:
            image.seek(0)
            image = ImageOps.exif_transpose(image).convert("RGB")
            if not self.native_resolution:
                image = ImageOps.fit(image, (self.image_size, self.image_size), Image.Resampling.LANCZOS,
                                     centering=(0.5, 0.5))
            pixels = np.asarray(image, dtype=np.uint8).copy()
        with self._lock:
            self.counters["images"] += 1
        return pixels

    def stats(self):
        with self._lock:
            return dict(self.counters, open_shards=len(self._fds))

    def close(self):
        with self._lock:
            for fd in self._fds.values():
                os.close(fd)
            self._fds.clear()
