"""Failure detection on the host (no GPU fault, trap or hang is ever provoked).

A sender and its receivers run in one process (threads) over the real control plane:
uvicorn + FastAPI controller, ZMQ worker thread, TCPStore session, gloo payload path.
Each test injects one failure and checks that it surfaces as a clear error well before
the configured deadline, instead of a hang.
"""
import socket
import threading
import time

import pytest
import torch

from weightbridge_b200 import TransferConfig, WeightData, WeightReceiver, WeightReceiverController, WeightSender
from weightbridge_b200.control.controller import ControllerError
from weightbridge_b200.control.sender import TransferError
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class Rollout:
    """FastAPI server + controller + one receiver worker, in this process."""

    def __init__(self, cfg, state_dict=None, meta=None, workers=1, make_receiver=True, model="tiny-llama",
                 layout=None):
        import uvicorn
        from fastapi import FastAPI
        arch = get_arch(model)
        self.lay = SGLangLayout(arch, **(layout or dict(tp=1)))
        self.params = self.lay.allocate(dtype=torch.float32)
        m, views = self.lay.to_wb(self.params)
        self.meta = meta or m
        app = FastAPI()
        self.ctl = WeightReceiverController(app, worker_num=workers, timeout_s=2.0)
        self.recv = None
        if make_receiver:
            self.recv = WeightReceiver(self.ctl.ipc_name, 0, self.meta,
                                       state_dict=views if state_dict is None else state_dict, config=cfg)
        port = _port()
        self.server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
        threading.Thread(target=self.server.run, daemon=True).start()
        t0 = time.time()
        while not self.server.started and time.time() - t0 < 20:
            time.sleep(0.02)
        self.url = f"http://127.0.0.1:{port}"

    def close(self):
        if self.recv is not None:
            self.recv.stop()
        self.server.should_exit = True
        self.ctl.close()


def _sender(cfg):
    lay = MegatronLayout(get_arch("tiny-llama"), tp=1)
    params = lay.allocate(dtype=torch.float32)
    meta, views = lay.to_wb(params)
    return lay, params, meta, views


def _cfg(**kw):
    base = dict(mode="cpu_direct", connect_timeout_s=30, sync_timeout_s=30, http_timeout_s=10)
    base.update(kw)
    return TransferConfig(**base)


@pytest.mark.parametrize("mode,direction", [("cpu_direct", "push"), ("gpu_direct", "push"), ("gpu_direct", "pull")])
def test_sync_then_receiver_never_updates_times_out(mode, direction):
    """gpu_direct with host tensors in one process runs the device protocol (work tables,
    flags, ready/done, status) through the C++ executor.  Pulling, the sender does not wait
    for the worker to be ready; it fails waiting for the worker to pull."""
    cfg = _cfg(sync_timeout_s=2.0, mode=mode, direction=direction)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender(mode, [ro.url], config=cfg)
        s.connect(meta)
        # one good sync first
        th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
        th.start()
        s.send(views)
        th.join(20)
        exp = ro.lay.allocate(dtype=torch.float32, fill=True)
        assert all(torch.equal(ro.params[n], exp[n]) for n in exp)
        assert ro.recv.epoch == 1
        if mode == "gpu_direct":
            pushed = direction == "push"      # pulling, the worker copies and no flag is written
            assert int(ro.recv.flags[0]) == (1 if pushed else 0)
            # a second good sync with new weights
            lay.fill(params, seed=5)
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            st = s.send(views)
            th.join(20)
            assert st.epoch == 2 and st.status == 0 and int(ro.recv.flags[0]) == (2 if pushed else 0)
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=5)
            assert all(torch.equal(ro.params[n], exp[n]) for n in exp)
        # now nobody calls request_update: send must fail by the deadline, not hang
        t0 = time.time()
        with pytest.raises(TransferError, match="ready" if direction == "push" else "pull"):
            s.send(views)
        assert time.time() - t0 < 10
    finally:
        ro.close()


def test_receiver_join_failure_reaches_sender_fast():
    cfg = _cfg(connect_timeout_s=60)
    # the receiver's state_dict lacks one entry: binding fails inside the worker's join
    arch = get_arch("tiny-llama")
    lay = SGLangLayout(arch, tp=1)
    params = lay.allocate(dtype=torch.float32)
    meta, views = lay.to_wb(params)
    views.pop("model.norm.weight")
    ro = Rollout(cfg, state_dict=views, meta=meta)
    try:
        _, _, smeta, _ = _sender(cfg)
        s = WeightSender("cpu_direct", [ro.url], config=cfg)
        t0 = time.time()
        with pytest.raises(Exception, match="model.norm.weight"):
            s.connect(smeta)
        assert time.time() - t0 < 15, "sender should learn of the failure long before the 60 s deadline"
        assert ro.recv.state.value == "failed"
    finally:
        ro.close()


def test_plan_digest_mismatch_is_detected(monkeypatch):
    import weightbridge_b200.control.receiver as rmod
    monkeypatch.setattr(rmod, "plan_digest", lambda ov: "corrupted")
    cfg = _cfg(connect_timeout_s=60)
    ro = Rollout(cfg)
    try:
        _, _, smeta, _ = _sender(cfg)
        s = WeightSender("cpu_direct", [ro.url], config=cfg)
        t0 = time.time()
        with pytest.raises(Exception, match="digest mismatch"):
            s.connect(smeta)
        assert time.time() - t0 < 15
    finally:
        ro.close()


def test_controller_gather_times_out_on_missing_worker():
    cfg = _cfg()
    ro = Rollout(cfg, workers=2)      # two workers expected, one exists
    try:
        t0 = time.time()
        with pytest.raises(ControllerError):
            ro.ctl._query_receivers_metadata()
        assert time.time() - t0 < 5
    finally:
        ro.close()


def test_controller_query_metadata_two_workers():
    """The reference's controller test, on the API it expected (worker_num kwarg and a
    synchronous _query_receivers_metadata), with two workers and empty metadata."""
    ctl = WeightReceiverController(None, worker_num=0)
    ctl.set_worker_num(2)
    empty = WeightData(meta_dict={})
    r0 = WeightReceiver(ctl.ipc_name, 0, empty)
    r1 = WeightReceiver(ctl.ipc_name, 1, empty)
    try:
        res = ctl._query_receivers_metadata()
        assert [r["rank"] for r in res] == [0, 1]
        assert all(r["metadata"] == {} for r in res)
    finally:
        r0.stop()
        r1.stop()
        ctl.close()


def test_update_without_arm_returns_false_and_stop_is_clean():
    cfg = _cfg()
    ro = Rollout(cfg)
    try:
        assert ro.recv.request_update() is False
        t0 = time.time()
        assert ro.recv.request_update(timeout=0.5) is False
        assert 0.4 < time.time() - t0 < 5
    finally:
        ro.close()
    assert not ro.recv.receiver_thread.is_alive()


def test_receive_request_rejected_before_connect():
    cfg = _cfg()
    ro = Rollout(cfg)
    try:
        import requests
        r = requests.post(f"{ro.url}/wbridge/receive", timeout=5)
        assert r.json()["status"] == "error"
        stats = requests.get(f"{ro.url}/wbridge/stats", timeout=5).json()
        assert stats[0]["state"] == "disconnected"
    finally:
        ro.close()


def test_connect_from_another_protocol_version_is_refused():
    """A sender of another protocol version (here: one that sends none) is refused at
    connect, before any session state is touched."""
    cfg = _cfg()
    ro = Rollout(cfg)
    try:
        import requests
        r = requests.post(f"{ro.url}/wbridge/connect", timeout=5, json={
            "master_address": "127.0.0.1", "master_port": 1, "base_rank": 1, "world_size": 2,
            "group_name": "wbridge", "sender_world_size": 1, "backend": "cpu_direct"})
        body = r.json()
        assert body["status"] == "error" and "protocol" in body["detail"][0]
        assert ro.recv.state.value == "disconnected"
    finally:
        ro.close()


@pytest.mark.parametrize("mode", ["cpu_direct", "gpu_direct"])
def test_resume_after_receiver_restart(mode):
    """A rollout worker restarts (new process state, new tensors): the sender reconnects and
    the next sync lands in the new worker's memory."""
    cfg = _cfg(mode=mode)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender(mode, [ro.url], config=cfg)
        s.connect(meta)
        th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
        th.start()
        s.send(views)
        th.join(20)
        # the worker dies and comes back with fresh (zeroed) parameters under the same rank
        ro.recv.stop()
        fresh = ro.lay.allocate(dtype=torch.float32)
        m2, v2 = ro.lay.to_wb(fresh)
        ro.recv = WeightReceiver(ro.ctl.ipc_name, 0, m2, state_dict=v2, config=cfg)
        time.sleep(0.2)
        s.reconnect()
        lay.fill(params, seed=9)
        th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
        th.start()
        st = s.send(views)
        th.join(20)
        assert st.epoch == 1
        exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=9)
        assert all(torch.equal(fresh[n], exp[n]) for n in exp)
    finally:
        ro.close()


@pytest.mark.parametrize("mode", ["cpu_direct", "gpu_direct"])
def test_reference_style_receiver_gets_tensors_at_update(mode):
    """The reference's flow: WeightReceiver(controller_ipc_name, rank, metadata) without
    tensors; the scheduler hands its state_dict to request_update."""
    cfg = _cfg(mode=mode)
    ro = Rollout(cfg, make_receiver=False)
    try:
        ro.recv = WeightReceiver(ro.ctl.ipc_name, 0, ro.meta, config=cfg)
        _, views = ro.lay.to_wb(ro.params)
        lay, params, meta, sviews = _sender(cfg)
        s = WeightSender(mode, [ro.url], config=cfg)
        s.connect(meta)
        for step in range(2):
            if step:
                lay.fill(params, seed=step)
            th = threading.Thread(target=lambda: ro.recv.request_update(views, timeout=20))
            th.start()
            s.send(sviews)
            th.join(20)
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=step)
            assert all(torch.equal(ro.params[n], exp[n]) for n in exp), step
    finally:
        ro.close()


def test_pull_direction_in_process():
    """direction='pull': the receiver loads the copies from the sender's memory (host path in
    one process), two syncs with new weights, sender waits until the receiver pulled."""
    cfg = _cfg(mode="gpu_direct", direction="pull")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        for step in range(2):
            if step:
                lay.fill(params, seed=step)
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            st = s.send(views)
            th.join(20)
            assert st.status == 0 and s.program is None          # nothing pushed: no quantised blocks
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=step)
            assert all(torch.equal(ro.params[n], exp[n]) for n in exp), step
        assert ro.recv.pull_program is not None and len(ro.recv.pull_program.tables) > 0
        # where the pulled bytes come from: one route per sender, summing to the program's stores
        routes = ro.recv.routes()
        assert len(routes) == 1 and not routes[0]["multicast"] and routes[0]["src"] == -1
        assert sum(r["bytes"] for r in routes) == ro.recv.pull_program.bytes_written > 0
        assert s.routes() == [] and s.delivered_bytes == 0            # the sender pushed nothing
        # other tensors (a second copy of the weights), then the first ones again: each switch
        # publishes the sender's memory anew and the receiver pulls from the right one
        params2 = lay.allocate(dtype=torch.float32, seed=7)
        _m2, views2 = lay.to_wb(params2)
        for vs, seed in ((views2, 7), (views, 1)):
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            s.send(vs)
            th.join(20)
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=seed)
            assert all(torch.equal(ro.params[n], exp[n]) for n in exp), seed
    finally:
        ro.close()


def test_pull_request_with_fp8_blocks_pushes_everything():
    """A session whose workers hold fp8 block-quantised entries pushes every copy even when
    pull was asked for: the sender quantises (halving the bytes on the link), and pulling the
    plain copies could only start after its kernel stored the blocks."""
    import uvicorn
    from fastapi import FastAPI
    cfg = _cfg(mode="gpu_direct", direction="pull")
    arch = get_arch("tiny-qwen3-moe")
    rl = SGLangLayout(arch, tp=1, quant="fp8_experts")
    rparams = rl.allocate(dtype=torch.bfloat16)
    rmeta, rviews = rl.to_wb(rparams)
    app = FastAPI()
    ctl = WeightReceiverController(app, worker_num=1, timeout_s=5)
    recv = WeightReceiver(ctl.ipc_name, 0, rmeta, state_dict=rviews, config=cfg)
    port = _port()
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    threading.Thread(target=server.run, daemon=True).start()
    while not server.started:
        time.sleep(0.02)
    try:
        ml = MegatronLayout(arch, ep=1)
        sparams = ml.allocate(dtype=torch.bfloat16)
        smeta, sviews = ml.to_wb(sparams)
        s = WeightSender("gpu_direct", [f"http://127.0.0.1:{port}"], config=cfg)
        s.connect(smeta)
        th = threading.Thread(target=lambda: recv.request_update(timeout=20))
        th.start()
        s.send(sviews)
        th.join(20)
        assert s.direction == "push" and recv.direction == "push"
        assert s.program is not None and len(s.program.tables.qwork) > 0 and len(s.program.tables.items) > 0
        assert recv.pull_program is None
        exp = rl.allocate(dtype=torch.bfloat16, fill=True)
        u8 = lambda t: t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t
        assert all(torch.equal(u8(rparams[n]), u8(exp[n])) for n in exp)
    finally:
        recv.stop()
        server.should_exit = True
        ctl.close()


@pytest.mark.parametrize("arm", ["direct", "http"])
@pytest.mark.parametrize("mode", ["cpu_direct", "gpu_direct"])
def test_both_arm_channels_sync(mode, arm):
    """A sync is armed either by one ZMQ message per worker (default) or by the reference's
    POST /wbridge/receive; both land the same weights and the controller sees the epochs."""
    cfg = _cfg(mode=mode, arm=arm)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender(mode, [ro.url], config=cfg)
        s.connect(meta)
        assert (s._arm_sock is not None) == (arm == "direct")
        for step in range(3):
            lay.fill(params, seed=step)
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            st = s.send(views, version=100 + step)
            th.join(20)
            assert st.epoch == step + 1
            assert ro.recv.weights_version == 100 + step          # the tag travels with the weights
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=step)
            assert all(torch.equal(ro.params[n], exp[n]) for n in exp), step
        stats = ro.ctl.get_stats()[0]
        assert stats["epoch"] == 3 and stats["weights_version"] == 102
        # a repeated arm of the pending epoch is harmless
        if arm == "direct":
            s._arm(4)
            s._arm(4)
            time.sleep(0.2)
            assert ro.recv.state.value == "awaiting_scheduler_update"
    finally:
        ro.close()


def test_direct_arm_to_a_stopped_worker_fails_fast():
    """The worker's process side is gone (its sockets closed): the arm is unroutable and the
    sync fails at once instead of waiting for the ready deadline."""
    cfg = _cfg(mode="gpu_direct", sync_timeout_s=20.0)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        ro.recv.stop()
        ro.recv = None
        time.sleep(0.5)              # the sender's connection sees the peer close
        t0 = time.time()
        with pytest.raises(TransferError, match="unreachable"):
            s.send(views)
        assert time.time() - t0 < 5
    finally:
        ro.close()


def test_sync_over_this_hosts_address():
    """The session store and the arm channel on the host's routable address instead of
    loopback (the disaggregated set-up: the receivers publish that address for their arm
    sockets, bound on every interface)."""
    from weightbridge_b200.control.session import local_address
    addr = local_address()
    if addr.startswith("127."):
        pytest.skip("no routable address on this host")
    cfg = _cfg(mode="cpu_direct", master_address=addr)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("cpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
        th.start()
        s.send(views)
        th.join(20)
        assert ro.recv._arm_sock.getsockopt_string(__import__("zmq").LAST_ENDPOINT).startswith("tcp://0.0.0.0:")
        exp = ro.lay.allocate(dtype=torch.float32, fill=True)
        assert all(torch.equal(ro.params[n], exp[n]) for n in exp)
    finally:
        ro.close()


def _cut(watch):
    """A process dying: its liveness connections close without the orderly bye."""
    import socket as _s
    watch._stop.set()
    watch._thread.join(2)
    for sock in list(watch._conns):
        try:
            sock.shutdown(_s.SHUT_RDWR)
        except OSError:
            pass
        sock.close()


def test_sender_dying_mid_sync_fails_the_receiver_at_once():
    """The receiver is waiting for a sender's done key when the sender's process goes away:
    the liveness connection closes without a bye and the wait ends with an error in well
    under the 30 s sync deadline."""
    from weightbridge_b200.control.receiver import ReceiveError
    cfg = _cfg(mode="gpu_direct", sync_timeout_s=30.0)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        out = {}

        def update():
            t0 = time.time()
            try:
                ro.recv.request_update(timeout=20)
                out["r"] = ("ok", time.time() - t0)
            except ReceiveError as e:
                out["r"] = (str(e), time.time() - t0)

        th = threading.Thread(target=update)
        th.start()
        s._arm(1)                                    # armed; the sender never launches
        b = s._board                                 # peers on one host: the handshake words
        assert b is not None
        b.wait([b.ready_slot(min(s.targets))], 1, 10.0, lambda: None, "the worker's ready")
        _cut(s._watch)
        th.join(20)
        msg, dt = out["r"]
        assert "left the session" in msg and dt < 10, out
    finally:
        ro.close()


def test_receiver_dying_while_a_sender_waits_for_ready():
    """The sender waits for a worker's ready key when the worker's process goes away: the
    send fails at once instead of at the 30 s deadline."""
    cfg = _cfg(mode="gpu_direct", sync_timeout_s=30.0)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        threading.Timer(0.5, lambda: _cut(ro.recv._watch)).start()   # nobody calls request_update
        t0 = time.time()
        with pytest.raises(TransferError, match="left the session"):
            s.send(views)
        assert time.time() - t0 < 10
    finally:
        ro.close()


def test_orderly_disconnect_is_not_a_loss():
    cfg = _cfg(mode="gpu_direct")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        watch = ro.recv._watch
        s.disconnect()
        time.sleep(0.5)
        assert watch.lost == []
    finally:
        ro.close()


@pytest.mark.parametrize("direction", ["push", "pull"])
def test_partial_sync_of_named_entries(direction):
    """send(names=...) moves only those entries (here: layer 0); the rest keeps the previous
    weights.  Alternating partial and full syncs reuses both compiled programs (pull: the
    worker's programs, selected by the subset digest in the senders' done values)."""
    cfg = _cfg(mode="gpu_direct", direction=direction)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        compiles = []
        orig = s._compile
        s._compile = lambda sd, sub=None: (compiles.append(sub), orig(sd, sub))[1]

        def sync(**kw):
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            s.send(views, **kw)
            th.join(20)

        sync()                                                   # everything at seed 0
        lay.fill(params, seed=1)
        layer0 = [n for n in meta.names() if n.startswith("model.layers.0.")]
        sync(names=layer0)
        exp0 = ro.lay.allocate(dtype=torch.float32, fill=True, seed=0)
        exp1 = ro.lay.allocate(dtype=torch.float32, fill=True, seed=1)
        # SGLang parameters of layer 0 (fused qkv / gate_up included) hold seed 1, the rest seed 0
        for n in exp0:
            want = exp1 if n.startswith("model.layers.0.") else exp0
            assert torch.equal(ro.params[n], want[n]), n
        lay.fill(params, seed=2)
        sync()
        sync(names=layer0)
        exp2 = ro.lay.allocate(dtype=torch.float32, fill=True, seed=2)
        assert all(torch.equal(ro.params[n], exp2[n]) for n in exp2)
        assert len(compiles) == 2                               # full + layer 0, each once
        if direction == "pull":
            assert len(ro.recv._pull_progs) == 2
    finally:
        ro.close()


def test_auto_transfer_mode_picks_cpu_direct_for_host_tensors():
    """transfer_mode="auto": rank 0 picks the mode from where the tensors live (here: host
    tensors, so cpu_direct) and every rank uses it."""
    cfg = _cfg(mode="cpu_direct")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("auto", [ro.url], config=_cfg(mode="auto"))
        s.connect(meta)
        assert s.config.mode == "cpu_direct"
        th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
        th.start()
        s.send(views)
        th.join(20)
        exp = ro.lay.allocate(dtype=torch.float32, fill=True)
        assert all(torch.equal(ro.params[n], exp[n]) for n in exp)
    finally:
        ro.close()


def test_controller_serves_its_own_http_server():
    """WeightReceiverController.serve(): a rollout process without a FastAPI app of its own."""
    from weightbridge_b200 import WeightReceiverController
    cfg = _cfg(mode="cpu_direct")
    arch = get_arch("tiny-llama")
    lay = SGLangLayout(arch, tp=1)
    params = lay.allocate(dtype=torch.float32)
    meta, views = lay.to_wb(params)
    with WeightReceiverController(worker_num=1, timeout_s=5) as ctl:
        url = ctl.serve()
        with WeightReceiver(ctl.ipc_name, 0, meta, state_dict=views, config=cfg) as recv:
            _l, sp, smeta, sviews = _sender(cfg)
            with WeightSender("cpu_direct", [url], config=cfg) as s:
                s.connect(smeta)
                th = threading.Thread(target=lambda: recv.request_update(timeout=20))
                th.start()
                s.send(sviews)
                th.join(20)
    exp = lay.allocate(dtype=torch.float32, fill=True)
    assert all(torch.equal(params[n], exp[n]) for n in exp)


def test_worker_endpoints_use_the_host_address_not_the_master_override(monkeypatch):
    """WBRIDGE_MASTER_ADDRESS names the sender's session store; a worker publishes its own
    address (WBRIDGE_HOST_ADDRESS) for its arm and liveness endpoints."""
    from weightbridge_b200.control.session import host_address, local_address
    monkeypatch.setenv("WBRIDGE_MASTER_ADDRESS", "10.1.2.3")
    monkeypatch.setenv("WBRIDGE_HOST_ADDRESS", "10.9.9.9")
    assert local_address() == "10.1.2.3" and host_address() == "10.9.9.9"
    monkeypatch.delenv("WBRIDGE_MASTER_ADDRESS")
    assert local_address() == "10.9.9.9"


def test_push_alternating_tensor_sets_uses_cached_programs():
    """Two sets of trainer tensors sent alternately: each send moves the set it is given, and
    each set's program is compiled once."""
    cfg = _cfg(mode="gpu_direct", direction="push")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        params2 = lay.allocate(dtype=torch.float32, seed=7)
        _m2, views2 = lay.to_wb(params2)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        compiles = []
        orig = s._compile
        s._compile = lambda sd, sub=None: (compiles.append(1), orig(sd, sub))[1]
        for vs, seed in ((views, 0), (views2, 7), (views, 0), (views2, 7)):
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            s.send(vs)
            th.join(20)
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=seed)
            assert all(torch.equal(ro.params[n], exp[n]) for n in exp), seed
            # one unicast route per receiver, summing to the program's stores (kept with each
            # cached program)
            routes = s.routes()
            assert len(routes) == 1 and routes[0]["dst"] == [-1] and not routes[0]["multicast"]
            assert s.delivered_bytes == routes[0]["bytes"] == s.program.bytes_written > 0
        assert len(compiles) == 2
    finally:
        ro.close()


def test_send_async_overlaps_and_serialises():
    """send_async returns at once; the future yields the sync's stats; two async sends run
    one after the other in call order; disconnect waits for the one in flight."""
    cfg = _cfg(mode="gpu_direct")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        got = []

        def worker():
            for _ in range(2):
                ro.recv.request_update(timeout=20)
                got.append(ro.recv.weights_version)

        th = threading.Thread(target=worker)
        th.start()
        f1 = s.send_async(views, version=1)
        f2 = s.send_async(views, version=2)
        assert f1.result(timeout=20).epoch == 1 and f2.result(timeout=20).epoch == 2
        th.join(20)
        assert got == [1, 2]
        exp = ro.lay.allocate(dtype=torch.float32, fill=True)
        assert all(torch.equal(ro.params[n], exp[n]) for n in exp)
        s.disconnect()
    finally:
        ro.close()


def test_send_async_snapshot_lets_the_caller_update_at_once():
    """send_async(snapshot=True) syncs a copy taken at the call: the trainer overwrites its
    parameters right after the call and the worker still receives the old values; the
    snapshot buffers are reused while the tensors stay the same."""
    cfg = _cfg(mode="gpu_direct")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        got = []

        def worker():
            for _ in range(2):
                ro.recv.request_update(timeout=20)
                got.append((ro.recv.weights_version, {n: t.clone() for n, t in ro.params.items()}))

        th = threading.Thread(target=worker)
        th.start()
        f1 = s.send_async(views, version=1, snapshot=True)
        buf = s._snap
        lay.fill(params, seed=9)                  # the optimizer step, before the sync ran
        f2 = s.send_async(views, version=2, snapshot=True)
        lay.fill(params, seed=4)
        assert f1.result(timeout=20).epoch == 1 and f2.result(timeout=20).epoch == 2
        th.join(20)
        assert s._snap is buf
        assert [v for v, _p in got] == [1, 2]
        for (_v, recvd), seed in zip(got, (0, 9)):
            exp = ro.lay.allocate(dtype=torch.float32, fill=True, seed=seed)
            assert all(torch.equal(recvd[n], exp[n]) for n in exp), seed
        s.disconnect()
    finally:
        ro.close()


def test_uncovered_rollout_entries_warn_or_fail():
    """A rollout entry that no sender holds (here: lm_head, the trainer ties its embeddings)
    is reported at connect; require_full_coverage turns the warning into an error."""
    import dataclasses
    cfg = _cfg(mode="cpu_direct")
    ro = Rollout(cfg)
    try:
        tied = dataclasses.replace(get_arch("tiny-llama"), tie_embeddings=True)
        lay = MegatronLayout(tied, tp=1)
        params = lay.allocate(dtype=torch.float32)
        meta, views = lay.to_wb(params)
        s = WeightSender("cpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        assert s.uncovered == {1: ["lm_head.weight"]}
        s.disconnect()
        strict = _cfg(mode="cpu_direct", require_full_coverage=True)
        with pytest.raises(TransferError, match="lm_head"):
            WeightSender("cpu_direct", [ro.url], config=strict).connect(meta)
    finally:
        ro.close()


@pytest.mark.parametrize("mode", ["gpu_direct", "cpu_direct"])
def test_receiver_rebind_without_reconnect(mode):
    """The engine reallocates its parameters: rebind() hands the worker new tensors, the next
    update binds them and the senders follow (a new binding generation in the ready key)."""
    cfg = _cfg(mode=mode)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender(mode, [ro.url], config=cfg)
        s.connect(meta)

        def sync(seed):
            lay.fill(params, seed=seed)
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            s.send(views)
            th.join(20)

        sync(0)
        old = {n: t.clone() for n, t in ro.params.items()}
        fresh = ro.lay.allocate(dtype=torch.float32)
        _m, fviews = ro.lay.to_wb(fresh)
        ro.recv.rebind(fviews)
        sync(4)
        exp4 = ro.lay.allocate(dtype=torch.float32, fill=True, seed=4)
        assert all(torch.equal(fresh[n], exp4[n]) for n in exp4)            # new tensors got sync 2
        assert all(torch.equal(ro.params[n], old[n]) for n in old)          # old ones untouched
        sync(5)
        exp5 = ro.lay.allocate(dtype=torch.float32, fill=True, seed=5)
        assert all(torch.equal(fresh[n], exp5[n]) for n in exp5)
    finally:
        ro.close()


def test_two_models_share_one_rollout_app():
    """Two controllers (policy and a second model) on one FastAPI app under URL prefixes;
    each sender syncs its own model through its prefix."""
    import uvicorn
    from fastapi import FastAPI
    from weightbridge_b200 import WeightReceiverController
    cfg = _cfg(mode="cpu_direct")
    app = FastAPI()
    ctls, recvs, stores = [], [], []
    for prefix in ("/policy", "/critic"):
        ctl = WeightReceiverController(app, worker_num=1, timeout_s=5, prefix=prefix)
        lay = SGLangLayout(get_arch("tiny-llama"), tp=1)
        p = lay.allocate(dtype=torch.float32)
        m, v = lay.to_wb(p)
        recvs.append(WeightReceiver(ctl.ipc_name, 0, m, state_dict=v, config=cfg))
        ctls.append(ctl)
        stores.append((lay, p))
    port = _port()
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    threading.Thread(target=server.run, daemon=True).start()
    while not server.started:
        time.sleep(0.02)
    try:
        for k, prefix in enumerate(("/policy", "/critic")):
            lay, params, meta, views = _sender(cfg)
            lay.fill(params, seed=10 + k)
            s = WeightSender("cpu_direct", [f"http://127.0.0.1:{port}{prefix}"], config=cfg)
            s.connect(meta)
            th = threading.Thread(target=lambda r=recvs[k]: r.request_update(timeout=20))
            th.start()
            s.send(views)
            th.join(20)
            s.disconnect()
        for k, (rl, rp) in enumerate(stores):
            exp = rl.allocate(dtype=torch.float32, fill=True, seed=10 + k)
            assert all(torch.equal(rp[n], exp[n]) for n in exp), k
    finally:
        for r in recvs:
            r.stop()
        server.should_exit = True
        for c in ctls:
            c.close()


def test_metrics_route_counts_syncs_and_failures():
    """GET /wbridge/metrics: Prometheus text with per-worker counters (syncs, failures,
    bytes) and gauges (epoch, weights version, state) that follow the syncs."""
    import requests
    cfg = _cfg(mode="gpu_direct")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        for v in (5, 6):
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            s.send(views, version=v)
            th.join(20)
        r = requests.get(f"{ro.url}/wbridge/metrics", timeout=5)
        assert r.status_code == 200 and r.headers["content-type"].startswith("text/plain")
        vals = {}
        for line in r.text.splitlines():
            if line and not line.startswith("#"):
                key, val = line.rsplit(" ", 1)
                vals[key] = float(val)
        assert vals['wbridge_receiver_syncs_total{worker="0"}'] == 2
        assert vals['wbridge_receiver_sync_failures_total{worker="0"}'] == 0
        assert vals['wbridge_receiver_bytes_total{worker="0"}'] == 2 * ro.recv.expected_bytes > 0
        assert vals['wbridge_receiver_epoch{worker="0"}'] == 2
        assert vals['wbridge_receiver_weights_version{worker="0"}'] == 6
        assert vals['wbridge_receiver_state{worker="0",state="connected"}'] == 1
        assert "# TYPE wbridge_receiver_syncs_total counter" in r.text
        s.disconnect()
    finally:
        ro.close()


@pytest.mark.parametrize("chunk", [0, 48 << 10])
def test_partial_syncs_over_the_wire(chunk):
    """names= in a wire mode: the sender tags the epoch with the subset's digest, both sides cut
    the subset's chunks alike (on the full set's buffers), and only those entries change."""
    cfg = _cfg(mode="cpu_direct", wire_chunk_bytes=chunk)
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("cpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        layer1 = [n for n in views if n.startswith("model.layers.1.")]

        def sync(seed, names=None, version=None):
            lay.fill(params, seed=seed)
            th = threading.Thread(target=lambda: ro.recv.request_update(timeout=20))
            th.start()
            s.send(views, names=names, version=version)
            th.join(20)

        sync(0)
        sync(5, names=layer1, version=7)
        in_l1 = lambda n: 5 if n.startswith("model.layers.1.") else 0      # noqa: E731
        exp0, exp5 = (ro.lay.allocate(dtype=torch.float32, fill=True, seed=sd) for sd in (0, 5))
        for n in ro.params:
            assert torch.equal(ro.params[n], (exp5 if in_l1(n) == 5 else exp0)[n]), n
        assert ro.recv.weights_version == 7
        sync(6, names=layer1)                      # cached subset: no new wire set
        sync(8)
        exp8 = ro.lay.allocate(dtype=torch.float32, fill=True, seed=8)
        assert all(torch.equal(ro.params[n], exp8[n]) for n in ro.params)
        assert set(s._wire_sets) == {None, frozenset(layer1)} and len(ro.recv._wire_sets) == 2
        full, part = s._wire_sets[None], s._wire_sets[frozenset(layer1)]
        for p, (bufs, _items) in part.peers.items():
            assert [b.data_ptr() for b in bufs] == [b.data_ptr() for b in full.peers[p][0][:len(bufs)]]
        s.disconnect()
    finally:
        ro.close()


def test_wait_for_version_takes_updates_until_the_tag():
    """A scheduler that needs weights of at least step 3 takes the pending updates (versions
    1..3) and returns; waiting for a version no sender produces ends at its deadline."""
    from weightbridge_b200.control.receiver import ReceiveError
    cfg = _cfg(mode="gpu_direct")
    ro = Rollout(cfg)
    try:
        lay, params, meta, views = _sender(cfg)
        s = WeightSender("gpu_direct", [ro.url], config=cfg)
        s.connect(meta)
        got = []
        th = threading.Thread(target=lambda: got.append(ro.recv.wait_for_version(3, timeout=30, poll_s=0.5)))
        th.start()
        for v in (1, 2, 3):
            s.send(views, version=v)
        th.join(30)
        assert got == [3] and ro.recv.weights_version == 3
        sm = s.summary()
        assert sm["syncs"] == 3 and sm["host_ms"]["p50"] > 0 and sm["bytes_written"] > 0
        assert set(sm) >= {"device_ms", "wait_ready_ms", "gbs"}
        t0 = time.time()
        with pytest.raises(ReceiveError, match="waiting for 4"):
            ro.recv.wait_for_version(4, timeout=1.0, poll_s=0.3)
        assert time.time() - t0 < 5
        s.disconnect()
    finally:
        ro.close()
