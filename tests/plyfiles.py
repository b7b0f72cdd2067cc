"""PLY files for the PLY tests, written here with numpy (the layouts the reference reads:
crates/brush-serde/src/import.rs, ply_gaussian.rs, quant.rs). Test helpers only."""
from __future__ import annotations

import numpy as np

_TYPES = {np.dtype("i1"): "char", np.dtype("u1"): "uchar", np.dtype("i2"): "short", np.dtype("u2"): "ushort",
          np.dtype("i4"): "int", np.dtype("u4"): "uint", np.dtype("f4"): "float", np.dtype("f8"): "double"}


def ply_bytes(elements, fmt="binary_little_endian", comments=()):
    """elements: list of (name, structured numpy array). Returns the file bytes."""
    head = ["ply", f"format {fmt} 1.0"] + [f"comment {c}" for c in comments]
    for name, arr in elements:
        head.append(f"element {name} {len(arr)}")
        for f in arr.dtype.names:
            head.append(f"property {_TYPES[arr.dtype[f].newbyteorder('=')]} {f}")
    head.append("end_header")
    out = ("\n".join(head) + "\n").encode()
    for _, arr in elements:
        if fmt == "ascii":
            lines = []
            for row in arr:
                lines.append(" ".join(repr(float(v)) if arr.dtype[i].kind == "f" else str(int(v))
                                      for i, v in enumerate(row)))
            out += ("\n".join(lines) + ("\n" if lines else "")).encode()
        else:
            order = "<" if fmt == "binary_little_endian" else ">"
            out += arr.astype(arr.dtype.newbyteorder(order)).tobytes()
    return out


def splat_rows(n, degree=3, seed=0, extra=(), drop=()):
    """Standard 3DGS vertex rows with random values; `extra` adds (name, dtype, values)."""
    rng = np.random.default_rng(seed)
    rest = 3 * ((degree + 1) ** 2 - 1)
    names = ["x", "y", "z", "scale_0", "scale_1", "scale_2", "opacity", "rot_0", "rot_1", "rot_2", "rot_3",
             "f_dc_0", "f_dc_1", "f_dc_2"] + [f"f_rest_{k}" for k in range(rest)]
    names = [nm for nm in names if nm not in drop]
    dt = [(nm, "f4") for nm in names] + [(nm, d) for nm, d, _ in extra]
    arr = np.zeros(n, dtype=dt)
    for nm in names:
        arr[nm] = rng.normal(size=n).astype(np.float32)
    for nm, _, vals in extra:
        arr[nm] = vals
    return arr


def compressed_elements(n, sh_rest=0, seed=0):
    """SuperSplat compressed layout: chunk bounds per 256 rows, packed vertex words, u8 SH."""
    rng = np.random.default_rng(seed)
    nc = (n + 255) // 256
    bnames = ["min_x", "max_x", "min_y", "max_y", "min_z", "max_z", "min_scale_x", "max_scale_x", "min_scale_y",
              "max_scale_y", "min_scale_z", "max_scale_z", "min_r", "max_r", "min_g", "max_g", "min_b", "max_b"]
    chunk = np.zeros(nc, dtype=[(b, "f4") for b in bnames])
    for k in range(0, 18, 2):
        lo = rng.uniform(-2, 0, nc).astype(np.float32)
        chunk[bnames[k]] = lo
        chunk[bnames[k + 1]] = lo + rng.uniform(0.1, 3, nc).astype(np.float32)
    vert = np.zeros(n, dtype=[("packed_position", "u4"), ("packed_rotation", "u4"), ("packed_scale", "u4"),
                              ("packed_color", "u4")])
    for f in vert.dtype.names:
        vert[f] = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    # keep the packed alpha away from 0 and 255 (finite logits)
    vert["packed_color"] = (vert["packed_color"] & np.uint32(0xFFFFFF00)) | rng.integers(1, 255, n).astype(np.uint32)
    els = [("chunk", chunk), ("vertex", vert)]
    if sh_rest:
        sh = np.zeros(n, dtype=[(f"f_rest_{k}", "u1") for k in range(sh_rest)])
        for f in sh.dtype.names:
            sh[f] = rng.integers(0, 256, n).astype(np.uint8)
        els.append(("sh", sh))
    return els
