"""Tensor-parallel decode: a model split over `world` GPUs (one process per GPU)
must produce the oracle's greedy tokens, like the single-GPU model.

CPU tests cover the shard checks of the C-ABI and the handle exchange over a
gloo process group of two ranks; the GPU test runs 2, 4 and 8 ranks, one per GPU
(each skipped on a box with fewer GPUs), with bounded device waits, so a rank that
fails makes the others return an error instead of hanging."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from channel_b200 import _lib as L
from tests.model_util import ring_step_lists, small_config


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_arguments_rejected():
    lib = L.load()
    cfg = small_config().to_c()
    fake_ctx = C.c_void_p(16)  # never dereferenced: the argument checks come first
    h = C.c_void_p()
    assert lib.ch_model_create_synthetic_sharded(fake_ctx, C.byref(cfg), 1, 2, 2, C.byref(h)) == L.CH_EINVAL
    assert lib.ch_model_create_synthetic_sharded(fake_ctx, C.byref(cfg), 1, 0, 9, C.byref(h)) == L.CH_EINVAL
    # 2 kv heads do not split over 4 ranks
    assert lib.ch_model_create_synthetic_sharded(fake_ctx, C.byref(cfg), 1, 0, 4, C.byref(h)) == L.CH_EINVAL
    assert b"divide by world" in lib.ch_last_error()


class _FakeShard:
    def __init__(self, rank):
        self.rank = rank
        self.attached = None

    def exchange_handle(self):
        return bytes([self.rank + 1]) * L.CH_IPC_HANDLE_BYTES

    def attach_peers(self, handles):
        self.attached = handles


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    from channel_b200.engine import attach_tensor_parallel
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    gm = _FakeShard(rank)
    attach_tensor_parallel(gm)
    q.put((rank, [h[0] for h in gm.attached], [len(h) for h in gm.attached]))
    dist.barrier()
    dist.destroy_process_group()


def test_handle_exchange_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = {}
    for _ in range(2):
        rank, firsts, lens = q.get(timeout=120)
        got[rank] = (firsts, lens)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(2):
        assert got[rank][0] == [1, 2], "handles must arrive in rank order"
        assert got[rank][1] == [L.CH_IPC_HANDLE_BYTES] * 2


# ---------------------------------------------------------------------------
SEED = 5


def _tp_config(world):
    """the small test model; 4 and 8 ranks need 8 kv heads (one or two per rank)"""
    return small_config() if world <= 2 else small_config(num_attention_heads=16, num_key_value_heads=8)


def _tp_worker(rank, world, port, xs, plan, prompt, slots, n_prev, q):
    try:
        import torch.distributed as dist

        from channel_b200 import GpuContext, GpuModelContext, gpu_dispatch_forward_token, gpu_dispatch_prefill_batch
        from channel_b200.engine import attach_tensor_parallel
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        ctx = GpuContext.init(rank)
        cfg = _tp_config(world)
        gm = GpuModelContext.synthetic_sharded(ctx, cfg, SEED, rank, world)
        attach_tensor_parallel(gm)
        gm.zero_state()
        dist.barrier()
        host = []
        for x, (clock, slot, act, sli) in zip(xs, plan):
            tok, cands = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
            host.append((int(tok), [c.id for c in cands][:8], [float(c.val) for c in cands][:8]))
        # prefill (token by token through the decode kernel) + device-resident decode
        gm.zero_state()
        dist.barrier()
        cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, n_prev)
        first = int(cands[0].id)
        n = len(prompt)
        dplan = []
        from channel_b200 import DynamicRingBuffer
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        for c in range(n):
            for layer in range(cfg.num_hidden_layers):
                ring.activateSlot(layer, c)
        for i in range(6):
            dplan.append((n + i,) + tuple(ring_step_lists(ring, cfg, n + i)))
        gm.decode_plan(dplan)
        gm.decode_run(first, len(dplan))
        loop = [int(t) for t in gm.decode_tokens(len(dplan))]
        q.put((rank, host, first, loop, None))
        dist.barrier()
        gm.deinit()
        ctx.deinit()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, None, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_oracle(oracle, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from channel_b200 import DynamicRingBuffer
    cfg = _tp_config(world)
    w = oracle.SyntheticWeights(cfg, SEED)
    om = oracle.Model(cfg, w)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    xs, plan, ref = [], [], []
    tok = 17
    for clock in range(10):
        slot, act, sli = ring_step_lists(ring, cfg, clock)
        x = oracle.embed(w.embed, [tok], cfg.hidden_size)[0]
        rtok, rid, rvals = om.forward_token(x, clock, slot, act, sli)
        xs.append(x)
        plan.append((clock, slot, act, sli))
        ref.append((int(rtok), rid, rvals))
        tok = int(rtok)
    # prefill reference: the oracle's batched prefill, then greedy decode over the ring
    om2 = oracle.Model(cfg, w)
    N = 24
    prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, N).astype(np.uint32)
    pring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    prev = pring.getPrefillPrevSlots(0, 0, N)
    slots = np.concatenate([prev, [pring.getSlotIndex(c) for c in range(N)]]).astype(np.uint32)
    for c in range(N):
        for layer in range(cfg.num_hidden_layers):
            pring.activateSlot(layer, c)
    ptok, _, _ = om2.prefill(oracle.embed(w.embed, prompt, cfg.hidden_size), slots, 0, len(prev))
    loop_ref, t = [], int(ptok)
    for i in range(6):
        clock = N + i
        slot, act, sli = ring_step_lists(pring, cfg, clock)
        t, _, _ = om2.forward_token(oracle.embed(w.embed, [t], cfg.hidden_size)[0], clock, slot, act, sli)
        loop_ref.append(int(t))

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_tp_worker, args=(r, world, port, xs, plan, prompt, slots, len(prev), q))
          for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        rank, host, first, loop, err = q.get(timeout=600)
        res[rank] = (host, first, loop, err)
    for p in ps:
        p.join(timeout=120)
    for rank in range(world):
        host, first, loop, err = res[rank]
        assert err is None, f"rank {rank}: {err}"
        for step, ((gtok, gids, gvals), (rtok, rid, rvals)) in enumerate(zip(host, ref)):
            assert gtok == rtok, f"rank {rank}: greedy token diverged at step {step}"
            assert np.allclose(gvals, rvals[:8], rtol=1e-3, atol=1e-3)
        assert first == int(ptok), f"rank {rank}: prefill token"
        assert loop == loop_ref, f"rank {rank}: device-loop tokens after prefill"
    for rank in range(1, world):
        assert res[rank][0] == res[0][0]


# ---------------------------------------------------------------------------
# Failure detection: a rank that leaves between steps.  Rank 1 stops calling (its
# process and memory stay alive: nothing of it is in flight and its arena stays
# mapped), the peers learn of it only through the decode kernel's bounded waits:
# rank 0's next ch_forward_token must come back with CH_ETIMEOUT within the bound
# (2 s per wait, and a launch that gave up once stops waiting), and rank 0's
# context must still run work afterwards.  Host signalling is through queues; no
# NCCL and no multicast memory are involved.
def _leave_worker(rank, world, port, xs, plan, q_out, q_left, q_done):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import time

        import torch.distributed as dist

        from channel_b200 import GpuContext, GpuModelContext, gpu_dispatch_forward_token
        from channel_b200.engine import attach_tensor_parallel
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        ctx = GpuContext.init(rank)
        cfg = _tp_config(world)
        gm = GpuModelContext.synthetic_sharded(ctx, cfg, SEED, rank, world)
        attach_tensor_parallel(gm)
        gm.zero_state()
        dist.barrier()
        toks = []
        for x, (clock, slot, act, sli) in zip(xs[:3], plan[:3]):  # three steps together
            toks.append(int(gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)[0]))
        ctx.synchronize()
        dist.barrier()  # every rank is between steps: nothing in flight
        if rank == 1:
            q_left.put(1)  # leave: no further calls, memory kept until rank 0 is done
            q_done.get(timeout=300)
            gm.deinit()
            ctx.deinit()
            q_out.put((rank, toks, None, None, None))
            return
        q_left.get(timeout=120)
        x, (clock, slot, act, sli) = xs[3], plan[3]
        t0 = time.time()
        status = None
        try:
            gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
        except L.ChannelError as e:
            status = e.status
        elapsed = time.time() - t0
        # the context still works: a plain single-GPU call on it
        lib = L.load()
        flags = C.c_uint32(0)
        L.check(lib.ch_ctx_device_status(ctx.handle, C.byref(flags)))
        y = torch.empty(16, dtype=torch.float32, device="cuda")
        xx = torch.ones(64, dtype=torch.float32, device="cuda")
        tiles = torch.zeros(lib.ch_q4_tile_bytes(16, 64), dtype=torch.uint8, device="cuda")
        L.check(lib.ch_gemv_q4(ctx.handle, tiles.data_ptr(), 16, 64, xx.data_ptr(), y.data_ptr()))
        ctx.synchronize()
        usable = bool(torch.isfinite(y).all().item())
        q_done.put(1)
        q_out.put((rank, toks, status, elapsed, usable))
        # rank 0's arena was mapped by rank 1: it is freed only after rank 1 let go
        gm.deinit()
        ctx.deinit()
    except Exception as e:  # report instead of hanging the parent
        q_out.put((rank, None, None, None, repr(e)))


@pytest.mark.gpu
def test_tp_rank_leaving_makes_next_step_time_out(oracle):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    from channel_b200 import DynamicRingBuffer
    cfg = _tp_config(world)
    w = oracle.SyntheticWeights(cfg, SEED)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    xs, plan = [], []
    for clock, tok in enumerate([17, 3, 99, 5]):
        slot, act, sli = ring_step_lists(ring, cfg, clock)
        xs.append(oracle.embed(w.embed, [tok], cfg.hidden_size)[0])
        plan.append((clock, slot, act, sli))
    ctx = mp.get_context("spawn")
    q_out, q_left, q_done = ctx.Queue(), ctx.Queue(), ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_leave_worker, args=(r, world, port, xs, plan, q_out, q_left, q_done))
          for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        rank, toks, status, elapsed, usable = q_out.get(timeout=600)
        res[rank] = (toks, status, elapsed, usable)
    for p in ps:
        p.join(timeout=120)
    assert res[0][0] is not None, f"rank 0 failed: {res[0][3]}"
    assert res[1][0] is not None, f"rank 1 failed: {res[1][3]}"
    assert res[0][0] == res[1][0], "the steps taken together agree"
    _, status, elapsed, usable = res[0]
    assert status == L.CH_ETIMEOUT, f"rank 0 got {status}"
    assert elapsed < 20.0, f"the bounded waits took {elapsed:.1f} s"
    assert usable, "rank 0's context must still run work after the timeout"
