"""Generate tests/golden/layout_golden.json by importing the reference's own transport/layout.py.

Run where the reference tree is available (it is not needed afterwards):
    python tests/golden/make_golden.py --reference /path/to/sgl-afd-plugin
The reference module is loaded by file path (it imports nothing outside the standard library), so neither
sglang nor libcuda is needed.  The JSON holds, for a set of geometries covering every benchmark config and edge
cases, every offset the transport uses, plus doorbell known-answer vectors (including the seq wrap and the
out-of-range fields that must raise) and the invalid geometries the reference rejects.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

GEOMETRIES = [
    # (num_a, group, slots, n_max, hidden, topk, num_f)
    (1, 1, 2, 512, 1024, 2, 2),        # config 1 (CPU torch reference shape)
    (1, 1, 2, 16384, 7168, 8, 1),      # 1 GPU loopback / 1A1F
    (2, 1, 2, 16384, 7168, 8, 2),      # 2A2F
    (4, 1, 2, 16384, 7168, 8, 4),      # 4A4F
    (2, 1, 2, 16384, 7168, 8, 6),      # 2A6F
    (2, 1, 2, 16384, 7168, 8, 4),      # config 3 (2A4F, 2 slots)
    (4, 1, 2, 8192, 8192, 6, 4),       # config 4 (FP8 4A4F)
    (8, 2, 8, 131071, 7168, 8, 8),     # maximum sizes: n_max at the doorbell limit, 8 slots
    (3, 3, 1, 1, 8, 1, 1),             # minimum sizes, TP group of 3
    (6, 2, 3, 1000, 1000, 5, 3),       # nothing aligned
]

INVALID = [
    dict(num_a=0, group=1, slots=1, n_max=1, hidden=8, topk=1, num_f=1),
    dict(num_a=3, group=2, slots=1, n_max=1, hidden=8, topk=1, num_f=1),
    dict(num_a=1, group=1, slots=1, n_max=131072, hidden=8, topk=1, num_f=1),
    dict(num_a=1, group=1, slots=0, n_max=1, hidden=8, topk=1, num_f=1),
    dict(num_a=1, group=1, slots=1, n_max=1, hidden=8, topk=1, num_f=-2),
]

DOORBELLS = [
    # (seq, n_tokens, layer_id, epoch)
    (0, 1, 0, 1),
    (1, 16384, 3, 1),
    (0xFFFFFFFF, 131071, 1023, 31),
    (0x1_0000_0000, 7, 5, 2),       # seq wraps: only the low 32 bits are kept
    (0x1_2345_6789, 4097, 60, 17),
    (12345, 100, 512, 30),
]

BAD_DOORBELLS = [(1, 0, 0, 1), (1, 131072, 0, 1), (1, 1, 1024, 1), (1, 1, 0, 0), (1, 1, 0, 32), (1, 1, -1, 1)]


def load_layout(ref_root: str):
    path = os.path.join(ref_root, "python", "sgl_asap_plugin", "transport", "layout.py")
    spec = importlib.util.spec_from_file_location("ref_layout", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_layout"] = mod  # dataclasses resolves annotations through sys.modules
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ASAP_REFERENCE_DIR"), required="ASAP_REFERENCE_DIR" not in os.environ,
                    help="the reference checkout (or set ASAP_REFERENCE_DIR)")
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "layout_golden.json"))
    args = ap.parse_args()
    L = load_layout(args.reference)
    geos = []
    for t in GEOMETRIES:
        g = L.Geometry(*t)
        entry = {"geometry": g.as_dict()}
        for name in ("ids_off", "w_off", "region_bytes", "recv_bytes", "host_bytes", "flags_bytes", "seg_bytes",
                     "result_bytes"):
            entry[name] = getattr(g, name)
        entry["region_off"] = [[g.region_off(a, s) for s in range(g.slots)] for a in range(g.num_a)]
        entry["bell_off"] = [[g.bell_off(a, s) for s in range(g.slots)] for a in range(g.num_a)]
        entry["done_off"] = [[g.done_off(f, s) for s in range(g.slots)] for f in range(g.num_f)]
        entry["seg_off"] = [[g.seg_off(f, s) for s in range(g.slots)] for f in range(g.num_f)]
        geos.append(entry)
    invalid = []
    for d in INVALID:
        try:
            L.Geometry(**d)
            msg = None
        except ValueError as exc:
            msg = str(exc)
        invalid.append({"geometry": d, "error": msg})
    bells = []
    for seq, n, layer, epoch in DOORBELLS:
        word = L.pack_doorbell(seq, n, layer, epoch)
        bells.append({"args": [seq, n, layer, epoch], "word": word, "unpacked": list(L.unpack_doorbell(word))})
    bad = []
    for seq, n, layer, epoch in BAD_DOORBELLS:
        try:
            L.pack_doorbell(seq, n, layer, epoch)
            msg = None
        except ValueError as exc:
            msg = str(exc)
        bad.append({"args": [seq, n, layer, epoch], "error": msg})
    consts = {k: getattr(L, k) for k in ("ALIGN", "FLAG_STRIDE", "FLAGS_PAGE", "BELL_STRIDE", "ACT_BYTES",
                                          "ID_BYTES", "W_BYTES", "PROTO_VERSION", "SEQ_MASK", "MAX_TOKENS",
                                          "MAX_LAYER", "MAX_EPOCH")}
    out = {"source": "python/sgl_asap_plugin/transport/layout.py (reference, imported by file path)",
           "constants": consts, "geometries": geos, "invalid_geometries": invalid, "doorbells": bells,
           "bad_doorbells": bad}
    with open(args.out, "w") as fh:
        json.dump(out, fh, indent=1)
    print(f"wrote {args.out}: {len(geos)} geometries, {len(bells)} doorbells")


if __name__ == "__main__":
    main()
