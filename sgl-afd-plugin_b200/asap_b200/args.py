"""The ``--asap-*`` flags, unchanged, and the transport geometry they define.

Field names, defaults and meaning follow the reference's python/sgl_asap_plugin/srt/arg_groups/fields/asap.py:
14-92; ``transport_geometry`` and ``bootstrap_endpoints`` follow srt/server_args.py:198-214; ``check_values`` the
range checks of srt/arg_groups/asap_hook.py:107-149 (MAX_MICRO_BATCHES = 8, n_max <= 131071).  Without SGLang the
flags parse with argparse (``add_cli_args`` / ``from_cli_args``) and round-trip through ``ASAP_*`` environment
variables like the reference's launcher exports them (server_args.py:163-177).
"""

from __future__ import annotations

import argparse
import os
import re
from dataclasses import asdict, dataclass, fields
from typing import List, Optional, Tuple

from .transport.layout import MAX_TOKENS, Geometry

MAX_MICRO_BATCHES = 8
_ADDR_RE = re.compile(r"^.+:(\d+)$")


@dataclass
class Asap:
    asap_role: str = "null"  # "null" | "attn" | "ffn"
    asap_ffn_size: Optional[int] = None
    asap_bootstrap_addr: str = "127.0.0.1:9600"
    asap_transport_mem: str = "auto"  # "auto" | "ipc" | "fabric"
    asap_max_dispatch_tokens: int = 16384
    asap_max_micro_batches: int = 2
    asap_min_batch_tokens: int = 0
    asap_max_wait_ms: float = 50.0
    asap_tbo_min_tokens: int = 6144
    asap_ffn_cuda_graph_max_tokens: int = 0
    asap_attn_dp_size: Optional[int] = None
    asap_attn_base_replica: int = 0
    asap_attn_tp_size: Optional[int] = None


_CHOICES = {"asap_role": ("null", "attn", "ffn"), "asap_transport_mem": ("auto", "ipc", "fabric")}


def add_cli_args(parser: argparse.ArgumentParser) -> None:
    group = parser.add_argument_group("ASAP")
    for f in fields(Asap):
        flag = "--" + f.name.replace("_", "-")
        kind = {"Optional[int]": int, "int": int, "float": float, "str": str}[str(f.type)]
        group.add_argument(flag, dest=f.name, type=kind, default=f.default, choices=_CHOICES.get(f.name))


def from_cli_args(ns: argparse.Namespace) -> Asap:
    defaults = Asap()
    given = {f.name: getattr(ns, f.name) for f in fields(Asap)
             if getattr(ns, f.name, None) != getattr(defaults, f.name)}
    if given and given.get("asap_role", "null") == "null":
        flags = ", ".join("--" + n.replace("_", "-") for n in sorted(given))
        raise ValueError(f"{flags} given without --asap-role attn|ffn")
    args = Asap(**given)
    check_values(args)
    return args


_process_args: Optional[Asap] = None


def set_asap_args(args: Optional[Asap]) -> None:
    """Install this process's ASAP arguments (srt/server_args.py:88-90); None forgets them."""
    global _process_args
    _process_args = args


def get_asap_args() -> Asap:
    """This process's ASAP arguments: the installed ones, else those the launcher exported as ASAP_* environment
    variables (role "null" outside an ASAP deployment; srt/server_args.py:93-97)."""
    global _process_args
    if _process_args is None:
        _process_args = from_env()
    return _process_args


def export_env(args: Asap) -> None:
    for f in fields(args):
        os.environ.pop(f.name.upper(), None)
        value = getattr(args, f.name)
        if value is not None:
            os.environ[f.name.upper()] = str(value)


def from_env() -> Asap:
    values = {}
    for f in fields(Asap):
        raw = os.environ.get(f.name.upper())
        if raw is None:
            continue
        kind = {"Optional[int]": int, "int": int, "float": float, "str": str}[str(f.type)]
        values[f.name] = kind(raw)
    return Asap(**values)


def check_values(args: Asap) -> None:
    """asap_hook.py:107-149."""
    m = _ADDR_RE.match(args.asap_bootstrap_addr)
    if not m or not 1 <= int(m.group(1)) <= 65535:
        raise ValueError(f"--asap-bootstrap-addr must be HOST:PORT, got {args.asap_bootstrap_addr!r}")
    if not 1 <= args.asap_max_dispatch_tokens <= MAX_TOKENS:
        raise ValueError(f"--asap-max-dispatch-tokens must be in [1, {MAX_TOKENS}], "
                         f"got {args.asap_max_dispatch_tokens}")
    if not 1 <= args.asap_max_micro_batches <= MAX_MICRO_BATCHES:
        raise ValueError(f"--asap-max-micro-batches must be in [1, {MAX_MICRO_BATCHES}], "
                         f"got {args.asap_max_micro_batches}")
    if not 0 <= args.asap_ffn_cuda_graph_max_tokens <= args.asap_max_dispatch_tokens:
        raise ValueError("--asap-ffn-cuda-graph-max-tokens must be in "
                         f"[0, --asap-max-dispatch-tokens {args.asap_max_dispatch_tokens}], "
                         f"got {args.asap_ffn_cuda_graph_max_tokens}")
    if args.asap_min_batch_tokens < 0 or args.asap_max_wait_ms < 0:
        raise ValueError("--asap-min-batch-tokens and --asap-max-wait-ms must be >= 0, got "
                         f"{args.asap_min_batch_tokens} and {args.asap_max_wait_ms}")
    if args.asap_tbo_min_tokens < 0:
        raise ValueError(f"--asap-tbo-min-tokens must be >= 0, got {args.asap_tbo_min_tokens}")
    for name in ("asap_ffn_size", "asap_attn_dp_size", "asap_attn_tp_size"):
        value = getattr(args, name)
        if value is not None and value < 1:
            raise ValueError(f"--{name.replace('_', '-')} must be >= 1, got {value}")
    if args.asap_role == "ffn" and None in (args.asap_attn_dp_size, args.asap_attn_tp_size):
        raise ValueError("--asap-role ffn needs --asap-attn-dp-size and --asap-attn-tp-size "
                         "(they size its receive buffers)")


def bootstrap_endpoints(args: Asap) -> List[Tuple[str, int]]:
    host, _, port = args.asap_bootstrap_addr.rpartition(":")
    return [(host, int(port) + f) for f in range(args.asap_ffn_size)]


def transport_geometry(args: Asap, hidden: int, topk: int) -> Geometry:
    return Geometry(num_a=args.asap_attn_dp_size * args.asap_attn_tp_size, group=args.asap_attn_tp_size,
                    slots=args.asap_max_micro_batches, n_max=args.asap_max_dispatch_tokens, hidden=hidden,
                    topk=topk, num_f=args.asap_ffn_size)


def as_dict(args: Asap) -> dict:
    return asdict(args)
