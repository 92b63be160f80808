"""AsapBuffer.connect(model_runner), the attention rank's bootstrap from the --asap-* flags (the reference's
srt/layers/moe/token_dispatcher/asap.py:99-147), end to end on CPU: two FfnServers listen on
--asap-bootstrap-addr's port + f, the buffer finds the model's AsapMoE layers, builds the geometry from the flags,
computes its A rank from the base replica and the DP / TP ranks, and connects over the real TCP handshake.  A
host-memory stand-in replaces the CUDA IPC arenas (no GPU)."""

import logging
import os
import socket
import tempfile
import types

import pytest
import torch

from asap_b200 import args as asap_args
from asap_b200.dispatcher import AsapBuffer
from asap_b200.layer import AsapMoE
from asap_b200.transport import channel as channel_mod
from asap_b200.transport.layout import HandshakeError
from asap_b200.transport.server import FfnServer
from host_mem import HostMem


def _free_port_pair():
    for _ in range(50):
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        with socket.socket() as s2:
            try:
                s2.bind(("127.0.0.1", port + 1))
                return port
            except OSError:
                continue
    raise RuntimeError("no two consecutive free ports")


class Model(torch.nn.Module):
    def __init__(self, layer_ids):
        super().__init__()
        self.blocks = torch.nn.ModuleList([AsapMoE(num_experts=16, hidden_size=256, intermediate_size=128,
                                                   layer_id=lid, top_k=2) for lid in layer_ids])


@pytest.fixture
def deployment(monkeypatch):
    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    port = _free_port_pair()
    flags = asap_args.Asap(asap_role="attn", asap_ffn_size=2, asap_bootstrap_addr=f"127.0.0.1:{port}",
                           asap_max_dispatch_tokens=64, asap_max_micro_batches=2, asap_attn_dp_size=2,
                           asap_attn_tp_size=1, asap_attn_base_replica=0)
    geometry = asap_args.transport_geometry(flags, 256, 2)
    model_fp = {"hidden": 256, "topk": 2, "n_experts": 16, "moe_layers": [1, 3]}
    servers = []
    for f in range(2):
        srv = FfnServer(f, geometry, device=0, run_dir=run_dir, host="127.0.0.1", port=port + f, model=model_fp,
                        info={"experts": [8 * f, 8 * f + 8], "quant_method": "mxfp4"})
        srv.mem = HostMem(run_dir)
        servers.append(srv.start())
    monkeypatch.setattr(channel_mod, "select_memory", lambda kind, device: HostMem(run_dir))
    monkeypatch.setenv("ASAP_DP_RANK", "1")
    monkeypatch.setenv("ASAP_TP_RANK", "0")
    asap_args.set_asap_args(flags)
    yield flags, geometry, servers
    asap_args.set_asap_args(None)
    buf = AsapBuffer._buffer
    if buf is not None:
        buf.channel.unmap_peers()
        AsapBuffer.install(None)
    for srv in servers:
        srv.unmap_peers()
    if buf is not None:
        buf.channel.close()
    for srv in servers:
        srv.close()


def test_connect_from_model_runner(deployment, caplog):
    flags, geometry, servers = deployment
    runner = types.SimpleNamespace(model=Model([3, 1]), gpu_id=0)
    with caplog.at_level(logging.INFO, logger="asap_b200.dispatcher"):
        buf = AsapBuffer.connect(runner)
    assert AsapBuffer.get() is buf
    ch = buf.channel
    assert ch.a == 1                                   # replica = base 0 + DP rank 1, TP size 1, TP rank 0
    assert ch.g == geometry and ch.endpoints == [("127.0.0.1", servers[0].port), ("127.0.0.1", servers[1].port)]
    assert ch.expert_bounds == [0, 8, 16]              # the equal split of n_experts over the F ranks
    assert ch.epochs == [1, 1]
    assert ch.hello["model"]["moe_layers"] == [1, 3]   # sorted by layer id
    for f, srv in enumerate(servers):
        assert 1 in srv.peers and srv.peers[1].epoch == 1
    assert buf.n_max == flags.asap_max_dispatch_tokens
    assert "attention rank 1 connected to 2 FFN ranks" in caplog.text
    assert "'experts': [8, 16]" in caplog.text and "mxfp4" in caplog.text


def test_connect_rejections(deployment):
    flags, geometry, servers = deployment
    with pytest.raises(RuntimeError, match="no AsapMoE layer"):
        AsapBuffer.connect(types.SimpleNamespace(model=torch.nn.Linear(2, 2), gpu_id=0))
    # a model the F ranks do not serve: the handshake's reason comes back
    wrong = types.SimpleNamespace(model=Model([1, 2]), gpu_id=0)
    with pytest.raises(HandshakeError, match="differ"):
        AsapBuffer.connect(wrong)
    assert AsapBuffer._buffer is None
