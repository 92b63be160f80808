"""What both sides of the A<->F transport agree on: arena layout, doorbell word, error types.

Byte-identical to the reference's python/sgl_asap_plugin/transport/layout.py (the wire contract between an
attention rank and an FFN rank): the same constants (layout.py:60-72), the same Geometry fields and offsets
(layout.py:115-198) and the same doorbell bits (layout.py:92-112):

    bits 0-31 seq | 32-48 n_tokens (1..MAX_TOKENS) | 49-58 layer_id (0..MAX_LAYER) | 59-63 epoch (1..MAX_EPOCH)

One difference in what the words mean, not in the bytes: a region of F rank f carries only the tokens routed
to one of f's experts (compacted, ascending token order), and the doorbell's n_tokens is that count.  F's
reply row j answers region row j; the A rank keeps the token -> row table and scatters in its combine kernel.
The CUDA library computes the same offsets (asap_geometry_offsets); the tests pin both to golden vectors
generated from the reference module.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, fields

ALIGN = 256
FLAG_STRIDE = 64
FLAGS_PAGE = 2 << 20
BELL_STRIDE = 64
ACT_BYTES = 2
ID_BYTES = 4
W_BYTES = 4

PROTO_VERSION = 4
SEQ_MASK = 0xFFFFFFFF
MAX_TOKENS = (1 << 17) - 1
MAX_LAYER = (1 << 10) - 1
MAX_EPOCH = (1 << 5) - 1


class TransportError(RuntimeError):
    """Base class of every transport failure."""


class HandshakeError(TransportError):
    """The peer could not be reached or rejected the connection."""


class ChannelPoisoned(TransportError):
    """A bounded device wait ran out; the slots stay unusable until reconnect()."""


def align_up(n: int, a: int = ALIGN) -> int:
    return -(-n // a) * a


def pack_doorbell(seq: int, n_tokens: int, layer_id: int, epoch: int) -> int:
    if not (1 <= n_tokens <= MAX_TOKENS and 0 <= layer_id <= MAX_LAYER and 1 <= epoch <= MAX_EPOCH):
        raise ValueError(
            f"doorbell field out of range: n_tokens={n_tokens} layer_id={layer_id} epoch={epoch}")
    return (seq & SEQ_MASK) | (n_tokens << 32) | (layer_id << 49) | (epoch << 59)


def unpack_doorbell(word: int):
    """-> (seq, n_tokens, layer_id, epoch)"""
    return word & SEQ_MASK, (word >> 32) & MAX_TOKENS, (word >> 49) & MAX_LAYER, word >> 59


@dataclass(frozen=True)
class Geometry:
    """Sizes of one deployment; A and F refuse to connect unless every field matches."""

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

    # F rank: RecvArena (device)
    @property
    def ids_off(self) -> int:
        return align_up(self.n_max * self.hidden * ACT_BYTES)

    @property
    def w_off(self) -> int:
        return self.ids_off + align_up(self.n_max * self.topk * ID_BYTES)

    @property
    def region_bytes(self) -> int:
        return self.w_off + align_up(self.n_max * self.topk * W_BYTES)

    @property
    def recv_bytes(self) -> int:
        return self.num_a * self.slots * self.region_bytes

    def region_off(self, a: int, s: int) -> int:
        return (a * self.slots + s) * self.region_bytes

    # F rank: doorbell page (host)
    @property
    def host_bytes(self) -> int:
        return align_up(self.num_a * self.slots * BELL_STRIDE, 4096)

    def bell_off(self, a: int, s: int) -> int:
        return (a * self.slots + s) * BELL_STRIDE

    # A rank: ResultArena (device)
    @property
    def flags_bytes(self) -> int:
        return align_up(self.num_f * self.slots * FLAG_STRIDE, FLAGS_PAGE)

    @property
    def seg_bytes(self) -> int:
        return align_up(self.n_max * self.hidden * ACT_BYTES)

    @property
    def result_bytes(self) -> int:
        return self.flags_bytes + self.num_f * self.slots * self.seg_bytes

    def done_off(self, f: int, s: int) -> int:
        return (f * self.slots + s) * FLAG_STRIDE

    def seg_off(self, f: int, s: int) -> int:
        return self.flags_bytes + (f * self.slots + s) * self.seg_bytes

    def as_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "Geometry":
        return cls(**{f.name: d[f.name] for f in fields(cls)})
