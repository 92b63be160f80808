"""Restatement of the reference's wire/arena contract (python/sgl_asap_plugin/transport/layout.py).

Test infrastructure only (see oracle/__init__.py).  Every number here must equal the reference's; the
golden vectors in tests/golden/layout_golden.json were produced by importing the reference module itself.
"""

from __future__ import annotations

from dataclasses import dataclass, fields

ALIGN = 256  # layout.py:60
FLAG_STRIDE = 64  # layout.py:61
FLAGS_PAGE = 2 << 20  # layout.py:62
BELL_STRIDE = 64  # layout.py:63
SEQ_MASK = 0xFFFFFFFF  # layout.py:69
MAX_TOKENS = (1 << 17) - 1  # layout.py:70
MAX_LAYER = (1 << 10) - 1  # layout.py:71
MAX_EPOCH = (1 << 5) - 1  # layout.py:72


def align_up(n: int, a: int = ALIGN) -> int:
    """layout.py:87-89."""
    return -(-n // a) * a


def pack_doorbell(seq: int, n_tokens: int, layer_id: int, epoch: int) -> int:
    """layout.py:92-102: bits 0-31 seq | 32-48 n | 49-58 layer | 59-63 epoch; out-of-range fields raise."""
    if not (1 <= n_tokens <= MAX_TOKENS and 0 <= layer_id <= MAX_LAYER and 1 <= epoch <= MAX_EPOCH):
        raise ValueError(f"doorbell field out of range: n_tokens={n_tokens} layer_id={layer_id} epoch={epoch}")
    return (seq & SEQ_MASK) | (n_tokens << 32) | (layer_id << 49) | (epoch << 59)


def unpack_doorbell(word: int):
    """layout.py:105-112."""
    return word & SEQ_MASK, (word >> 32) & MAX_TOKENS, (word >> 49) & MAX_LAYER, word >> 59


@dataclass(frozen=True)
class Geometry:
    """layout.py:115-198."""

    num_a: int
    group: int
    slots: int
    n_max: int
    hidden: int
    topk: int
    num_f: int

    def __post_init__(self):
        bad = [f"{f.name}={getattr(self, f.name)!r}" for f in fields(self)
               if not isinstance(getattr(self, f.name), int) or getattr(self, f.name) < 1]
        if not bad and self.num_a % self.group:
            bad.append(f"num_a={self.num_a} is not a multiple of group={self.group}")
        if not bad and self.n_max > MAX_TOKENS:
            bad.append(f"n_max={self.n_max} exceeds the {MAX_TOKENS} tokens a doorbell can announce")
        if bad:
            raise ValueError("invalid transport geometry: " + ", ".join(bad))

    @property
    def ids_off(self):
        return align_up(self.n_max * self.hidden * 2)

    @property
    def w_off(self):
        return self.ids_off + align_up(self.n_max * self.topk * 4)

    @property
    def region_bytes(self):
        return self.w_off + align_up(self.n_max * self.topk * 4)

    @property
    def recv_bytes(self):
        return self.num_a * self.slots * self.region_bytes

    def region_off(self, a, s):
        return (a * self.slots + s) * self.region_bytes

    @property
    def host_bytes(self):
        return align_up(self.num_a * self.slots * BELL_STRIDE, 4096)

    def bell_off(self, a, s):
        return (a * self.slots + s) * BELL_STRIDE

    @property
    def flags_bytes(self):
        return align_up(self.num_f * self.slots * FLAG_STRIDE, FLAGS_PAGE)

    @property
    def seg_bytes(self):
        return align_up(self.n_max * self.hidden * 2)

    @property
    def result_bytes(self):
        return self.flags_bytes + self.num_f * self.slots * self.seg_bytes

    def done_off(self, f, s):
        return (f * self.slots + s) * FLAG_STRIDE

    def seg_off(self, f, s):
        return self.flags_bytes + (f * self.slots + s) * self.seg_bytes
