"""The --asap-* flags (asap_b200.args): defaults as the reference declares them
(srt/arg_groups/fields/asap.py:14-92), CLI and environment round trips, the range checks
(srt/arg_groups/asap_hook.py:107-149), and the transport geometry the flags define (srt/server_args.py:198-214)."""

import argparse

import pytest

from asap_b200 import args as A
from asap_b200.transport.layout import MAX_TOKENS, Geometry

REFERENCE_DEFAULTS = {
    "asap_role": "null", "asap_ffn_size": None, "asap_bootstrap_addr": "127.0.0.1:9600",
    "asap_transport_mem": "auto", "asap_max_dispatch_tokens": 16384, "asap_max_micro_batches": 2,
    "asap_min_batch_tokens": 0, "asap_max_wait_ms": 50.0, "asap_tbo_min_tokens": 6144,
    "asap_ffn_cuda_graph_max_tokens": 0, "asap_attn_dp_size": None, "asap_attn_base_replica": 0,
    "asap_attn_tp_size": None,
}


def parse(argv):
    p = argparse.ArgumentParser()
    A.add_cli_args(p)
    return A.from_cli_args(p.parse_args(argv))


def test_defaults_match_reference():
    assert A.as_dict(A.Asap()) == REFERENCE_DEFAULTS
    assert A.as_dict(parse([])) == REFERENCE_DEFAULTS


def test_cli_round_trip_and_choices():
    a = parse(["--asap-role", "ffn", "--asap-ffn-size", "4", "--asap-attn-dp-size", "4", "--asap-attn-tp-size", "1",
               "--asap-max-dispatch-tokens", "8192", "--asap-max-micro-batches", "3", "--asap-max-wait-ms", "2.5",
               "--asap-transport-mem", "ipc"])
    assert (a.asap_role, a.asap_ffn_size, a.asap_max_dispatch_tokens, a.asap_max_micro_batches) == ("ffn", 4, 8192, 3)
    assert a.asap_max_wait_ms == 2.5 and a.asap_transport_mem == "ipc"
    with pytest.raises(SystemExit):  # argparse rejects a role outside the reference's Literal
        parse(["--asap-role", "both"])
    with pytest.raises(ValueError, match="without --asap-role"):
        parse(["--asap-ffn-size", "2"])


def test_env_round_trip(monkeypatch):
    for f in REFERENCE_DEFAULTS:
        monkeypatch.delenv(f.upper(), raising=False)
    a = A.Asap(asap_role="attn", asap_ffn_size=2, asap_max_dispatch_tokens=4096, asap_max_wait_ms=7.0,
               asap_attn_dp_size=2)
    A.export_env(a)
    try:
        assert A.from_env() == a
    finally:
        for f in REFERENCE_DEFAULTS:
            monkeypatch.delenv(f.upper(), raising=False)


@pytest.mark.parametrize("kw,msg", [
    ({"asap_bootstrap_addr": "localhost"}, "HOST:PORT"),
    ({"asap_bootstrap_addr": "h:0"}, "HOST:PORT"),
    ({"asap_bootstrap_addr": "h:65536"}, "HOST:PORT"),
    ({"asap_max_dispatch_tokens": 0}, "max-dispatch-tokens"),
    ({"asap_max_dispatch_tokens": MAX_TOKENS + 1}, "max-dispatch-tokens"),
    ({"asap_max_micro_batches": 0}, "max-micro-batches"),
    ({"asap_max_micro_batches": A.MAX_MICRO_BATCHES + 1}, "max-micro-batches"),
    ({"asap_ffn_cuda_graph_max_tokens": 16385}, "cuda-graph-max-tokens"),
    ({"asap_min_batch_tokens": -1}, "min-batch-tokens"),
    ({"asap_max_wait_ms": -0.5}, "max-wait-ms"),
    ({"asap_tbo_min_tokens": -1}, "tbo-min-tokens"),
    ({"asap_ffn_size": 0}, "ffn-size"),
    ({"asap_attn_tp_size": 0}, "attn-tp-size"),
    ({"asap_role": "ffn", "asap_attn_dp_size": 2}, "needs --asap-attn-dp-size and --asap-attn-tp-size"),
])
def test_range_checks(kw, msg):
    with pytest.raises(ValueError, match=msg):
        A.check_values(A.Asap(**kw))


def test_edges_accepted():
    A.check_values(A.Asap(asap_max_dispatch_tokens=MAX_TOKENS, asap_max_micro_batches=A.MAX_MICRO_BATCHES,
                          asap_ffn_cuda_graph_max_tokens=MAX_TOKENS, asap_bootstrap_addr="[::1]:65535"))


def test_geometry_and_endpoints():
    a = A.Asap(asap_role="ffn", asap_ffn_size=4, asap_attn_dp_size=4, asap_attn_tp_size=1,
               asap_bootstrap_addr="10.0.0.5:9600", asap_max_micro_batches=2, asap_max_dispatch_tokens=16384)
    A.check_values(a)
    assert A.transport_geometry(a, hidden=7168, topk=8) == Geometry(4, 1, 2, 16384, 7168, 8, 4)
    assert A.bootstrap_endpoints(a) == [("10.0.0.5", 9600 + f) for f in range(4)]
    tp2 = A.Asap(asap_role="ffn", asap_ffn_size=2, asap_attn_dp_size=2, asap_attn_tp_size=2)
    g = A.transport_geometry(tp2, hidden=1024, topk=2)
    assert (g.num_a, g.group) == (4, 2)  # one A rank per attention GPU, grouped by TP
