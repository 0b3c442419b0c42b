"""Minimal GGUF v3 tensor-table reader used by the tests to rewrite the data of
one tensor in place (for instance to give a synthetic NextN layer weights whose
drafts the target model accepts).  Test helper only."""
import struct

import numpy as np

_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}


class GGUF:
    def __init__(self, path):
        self.path = path
        with open(path, "rb") as f:
            buf = f.read()
        self._o = 0
        self._b = buf
        magic, version = struct.unpack_from("<II", buf, 0)
        assert magic == 0x46554747 and version == 3, "not a GGUF v3 file"
        self._o = 8
        n_tensors, n_kv = self._u64(), self._u64()
        self.kv = {}
        for _ in range(n_kv):
            k = self._str()
            self.kv[k] = self._value(self._u32())
        self.tensors = {}
        self.dim_offsets = {}
        for _ in range(n_tensors):
            name = self._str()
            nd = self._u32()
            self.dim_offsets[name] = [self._o + 8 * d for d in range(nd)]
            shape = [self._u64() for _ in range(nd)]
            typ = self._u32()
            off = self._u64()
            self.tensors[name] = (shape, typ, off)
        align = int(self.kv.get("general.alignment", 32))
        self.data_start = (self._o + align - 1) // align * align

    def _u32(self):
        v = struct.unpack_from("<I", self._b, self._o)[0]
        self._o += 4
        return v

    def _u64(self):
        v = struct.unpack_from("<Q", self._b, self._o)[0]
        self._o += 8
        return v

    def _str(self):
        n = self._u64()
        s = self._b[self._o:self._o + n].decode()
        self._o += n
        return s

    def _value(self, t):
        if t == 8:
            return self._str()
        if t == 9:
            et, n = self._u32(), self._u64()
            return [self._value(et) for _ in range(n)]
        fmt = "<" + _SCALAR[t]
        v = struct.unpack_from(fmt, self._b, self._o)[0]
        self._o += struct.calcsize(fmt)
        return v

    def set_dim(self, name, d, value):
        """Rewrites dimension d of tensor `name` in the tensor directory."""
        with open(self.path, "r+b") as f:
            f.seek(self.dim_offsets[name][d])
            f.write(struct.pack("<Q", value))

    def replace(self, name, data):
        """Overwrites the stored bytes of tensor `name` (same size)."""
        shape, typ, off = self.tensors[name]
        data = np.ascontiguousarray(data).view(np.uint8).ravel()
        n = int(np.prod(shape))
        want = {0: n * 4, 1: n * 2, 12: n // 256 * 144, 13: n // 256 * 176, 14: n // 256 * 210}[typ]
        assert data.size == want, (name, data.size, want)
        with open(self.path, "r+b") as f:
            f.seek(self.data_start + off)
            f.write(data.tobytes())
        return shape, typ
