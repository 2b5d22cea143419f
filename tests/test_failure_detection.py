"""Failure detection on gloo CPU ranks: a rank that raises or exits is detected by the others
on the host within a bounded time (no GPU involved, nothing faults or hangs a device)."""
import time

import pytest

from tests.dist_utils import run_ranks


def _loop(rank, world, kind):
    import torch
    import torch.distributed as dist

    from centrifuge_b200.utils.watchdog import FaultInjector, PeerFailure, Watchdog, failed_peers
    store = dist.distributed_c10d._get_default_store()
    wd = Watchdog(store, rank, world, interval=0.2, timeout=2.0)
    inj = FaultInjector(f"rank=1,step=2,kind={kind}", rank, wd.hb)
    t0 = time.time()
    x = torch.ones(4)
    try:
        for step in range(6):
            inj.at_step(step)
            wd.check()
            dist.all_reduce(x)
            time.sleep(0.3)
    except PeerFailure as e:
        return {"detected": e.ranks, "how": "watchdog", "secs": time.time() - t0}
    except RuntimeError as e:
        if rank == 1:
            wd.report(e)
            return {"failed_self": str(e)}
        # a collective that was in flight failed (peer gone or process-group timeout); the
        # store says who: a failure report, or a heartbeat that stops within its timeout
        deadline = time.time() + 10
        found = set()
        while not found and time.time() < deadline:
            found = {r for r, _ in failed_peers(store, world, rank)} | set(wd.hb.dead_peers())
            time.sleep(0.2)
        return {"detected": sorted(found), "how": "collective-error", "secs": time.time() - t0}
    finally:
        wd.close()
    return {"detected": [], "how": "none"}


@pytest.mark.parametrize("kind", ["raise", "exit"])
def test_peer_failure_detected(kind):
    res = run_ranks(_loop, 3, kind, timeout=120, pg_timeout=6, expect=3 if kind == "raise" else 2)
    survivors = [r for r in (0, 2)]
    for r in survivors:
        assert res[r]["detected"] == [1], res[r]
        assert res[r]["secs"] < 60
    if kind == "raise":
        assert "injected fault" in res[1]["failed_self"]


def test_checkpoint_corruption_detected(tmp_path):
    import torch

    from centrifuge_b200.utils.checkpoint import load_training_state, save_training_state
    save_training_state(str(tmp_path), 0, {"master": torch.randn(64)}, {"step": 1, "completed_steps": 1})
    p = tmp_path / "training_states" / "optim_rank0.pt"
    data = bytearray(p.read_bytes())
    data[len(data) // 2] ^= 0xFF
    p.write_bytes(bytes(data))
    with pytest.raises(RuntimeError, match="checksum"):
        load_training_state(str(tmp_path), 0)


def test_ref_client_survives_server_drop():
    import socket
    import threading

    from centrifuge_b200.data.ref_server import init_single_socket
    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(1)
    port = srv.getsockname()[1]

    def accept_and_drop():
        c, _ = srv.accept()
        c.close()  # the server drops the connection without answering

    threading.Thread(target=accept_and_drop, daemon=True).start()
    recv_q, send_q = init_single_socket("127.0.0.1", port)
    send_q.put([[1, 2, 3]])
    import queue
    with pytest.raises(queue.Empty):
        recv_q.get(timeout=2)
    srv.close()
