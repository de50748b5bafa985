"""Strata pack ingestion: crosslane's index over the model's GGUF shards.

A pack is ``<dir>/ds4.txt`` ("key value" lines: model_dir, format, geometry) and
``<dir>/tensors.txt`` ("file <i> <shard>", "t <name> <dtype> <file> <offset> <bytes>
<shape...>") (engine/strata/sycl/stage/wiring/weight_source.hpp:1-5,
pack_source.cpp:144-185). ``StrataPack`` reads one through the library
(``clb_strata_pack_*``: the reference's checks, pread of the stored bytes);
``ExpertBank.load_strata_pack`` repacks every matrix placed on a bank into the HBM layout;
``write_pack`` writes a single-shard pack (fixtures, converted checkpoints).
"""
import ctypes as C
import os

import numpy as np

from ._capi import ErrorV1, check, lib

ROLES = ("w1", "w3", "w2")  # gate, up, down


def expert_tensor(layer: int, expert: int, role: int) -> str:
    return f"layers.{layer}.ffn.experts.{expert}.{ROLES[role]}.weight"


class StrataPack:
    def __init__(self, directory: str):
        self._h = C.c_void_p()
        err = ErrorV1()
        check(lib.clb_strata_pack_open(os.fsencode(directory), C.byref(self._h), C.byref(err)), err)

    def close(self):
        if getattr(self, "_h", None):
            lib.clb_strata_pack_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def meta(self, key: str):
        buf = C.create_string_buffer(4096)
        rc = lib.clb_strata_pack_meta(self._h, key.encode(), buf, len(buf))
        return buf.value.decode() if rc == 0 else None

    def tensor(self, name: str):
        """-> (dtype, bytes, shape) or None."""
        dtype = C.create_string_buffer(64)
        nbytes = C.c_uint64(0)
        shape = (C.c_int64 * 8)()
        ndim = C.c_int32(0)
        rc = lib.clb_strata_pack_tensor(self._h, name.encode(), dtype, len(dtype), C.byref(nbytes), shape, 8,
                                        C.byref(ndim))
        if rc != 0:
            return None
        return dtype.value.decode(), int(nbytes.value), tuple(shape[i] for i in range(min(ndim.value, 8)))

    def read(self, name: str, offset: int = 0, nbytes: int = None) -> bytes:
        if nbytes is None:
            info = self.tensor(name)
            if info is None:
                raise KeyError(name)
            nbytes = info[1] - offset
        out = np.empty(nbytes, np.uint8)
        err = ErrorV1()
        check(lib.clb_strata_pack_read(self._h, name.encode(), offset, C.c_void_p(out.ctypes.data), nbytes,
                                       C.byref(err)), err)
        return out.tobytes()


def write_pack(directory: str, tensors, meta, shard: str = "model.gguf"):
    """tensors: iterable of (name, dtype, raw bytes, shape); meta: ds4.txt keys (model_dir
    defaults to the pack directory itself, format to "gguf")."""
    os.makedirs(directory, exist_ok=True)
    meta = {"model_dir": ".", "format": "gguf", **meta}
    lines, offset = [f"file 0 {shard}"], 0
    with open(os.path.join(directory, shard), "wb") as f:
        for name, dtype, raw, shape in tensors:
            f.write(raw)
            lines.append(f"t {name} {dtype} 0 {offset} {len(raw)} " + " ".join(str(int(d)) for d in shape))
            offset += len(raw)
    with open(os.path.join(directory, "tensors.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")
    with open(os.path.join(directory, "ds4.txt"), "w") as f:
        f.write("".join(f"{k} {v}\n" for k, v in meta.items()))
