"""1A1F on two GPUs (needs 2 GPUs; skipped otherwise): an A rank on GPU 0 and an F rank on GPU 1 in two
processes, connected by the TCP handshake and CUDA IPC; the dispatch kernels store over NVLink into the F rank's
RecvArena and ring its doorbell page, the F chain waits for the doorbell on its own GPU and stores the reply rows
and done flag into the A rank's ResultArena, the combine waits for them.  Output within relative L2 1e-2 of the
oracle, for several messages on both slots."""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, H, I, K, T = 8, 512, 256, 2, 200


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _proc(rank, port0, run_dir, q):
    try:
        import torch.distributed as dist

        from asap_b200.experts import Mxfp4Experts
        from asap_b200.transport.layout import Geometry

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port0))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        torch.cuda.set_device(rank)
        g = Geometry(1, 1, 2, 256, H, K, 1)
        experts = Mxfp4Experts.random(E, H, I, seed=5, device=f"cuda:{rank}")  # same bytes on both GPUs
        msgs = 4
        if rank == 1:
            from asap_b200.scheduler import FfnScheduler
            from asap_b200.transport.server import FfnServer

            srv = FfnServer(0, g, device=1, run_dir=run_dir, host="127.0.0.1", port=0).start()
            sched = FfnScheduler(srv, {0: experts}, timeout_s=30.0)
            obj = [srv.port]
            dist.broadcast_object_list(obj, src=1)
            dist.barrier()  # A connected
            stream = torch.cuda.current_stream()
            for m in range(msgs):  # queued before the messages arrive: each job waits for its doorbell
                sched.run_device_wait(0, m % 2, m // 2 + 1, 0, stream.cuda_stream)
            dist.barrier()  # A has its answers
            torch.cuda.synchronize()
            sched.check()
            dist.barrier()
            srv.unmap_peers()
            dist.barrier()
            sched.close()
            srv.close()
        else:
            from asap_b200.transport.channel import AttnChannel
            from oracle import moe, mx

            obj = [None]
            dist.broadcast_object_list(obj, src=1)
            ch = AttnChannel(0, g, [("127.0.0.1", obj[0])], device=0, expert_bounds=[0, E], timeout_s=30.0).connect()
            dist.barrier()
            gate, up = moe.dequant_w13(experts.w13.cpu().numpy(), experts.w13_sf.cpu().numpy(), E, H, I)
            w2 = moe.dequant_w2(experts.w2.cpu().numpy(), experts.w2_sf.cpu().numpy(), E, H, I)
            rng = np.random.default_rng(1)
            send = torch.cuda.Stream()
            stream = torch.cuda.current_stream()
            errs = []
            for m in range(msgs):
                x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
                ids, w = moe.topk_routing(rng.standard_normal((T, E)), K, "softmax")
                xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
                it, wt = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
                send.wait_stream(stream)
                t = ch.send(0, m % 2, xt.data_ptr(), it.data_ptr(), wt.data_ptr(), T, send.cuda_stream)
                out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
                ch.combine(t, out.data_ptr(), stream.cuda_stream)
                torch.cuda.synchronize()
                ch.check()
                ref = moe.round_trip(x, ids, w, [0, E], [(gate, up, w2)])
                errs.append(moe.rel_l2(out.float().cpu().numpy(), ref))
            dist.barrier()
            dist.barrier()
            ch.unmap_peers()
            dist.barrier()
            ch.close()
            q.put(("errs", errs))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # noqa: BLE001
        import traceback

        q.put(("error", f"rank {rank}: {exc!r}\n{traceback.format_exc()}"))
        raise


def test_one_a_one_f_on_two_gpus(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    run_dir = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port0 = _free_port()
    procs = [ctx.Process(target=_proc, args=(r, port0, run_dir, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    results = []
    while not q.empty():
        results.append(q.get())
    errors = [r[1] for r in results if r[0] == "error"]
    assert not errors, "\n".join(errors)
    errs = [r[1] for r in results if r[0] == "errs"][0]
    assert all(e < 1e-2 for e in errs), errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
