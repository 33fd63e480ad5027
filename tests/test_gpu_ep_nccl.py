"""Expert parallelism across real GPUs: one process per GPU (spawned), NCCL all-to-all exchanges through
moe_forward_ep, each rank holding its block of experts. Every rank's output must equal the single-GPU result for its
tokens bit for bit, through the torch.distributed orchestration (moe_forward_ep) and through the library's own NCCL
communicator (moe_forward_ep_native). Skipped with fewer than two GPUs (the emulated-rank test covers the kernels on
one GPU)."""
import datetime
import os
import socket
import tempfile
import time

import numpy as np
import pytest

from willow_v2_b200 import synth

pytestmark = pytest.mark.gpu
SEED, LAYER, TOKENS_PER_RANK = 0, 0, 1024


def _weights(moe, torch, ctx, zipf):
    return moe.LayerWeights(
        router_w=torch.from_numpy(synth.router_weight(SEED, LAYER)).cuda(),
        shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, LAYER)).cuda(),
        shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, LAYER, 256).reshape(-1)).cuda(),
        shared_down=torch.from_numpy(synth.expert_down(SEED, LAYER, 256).reshape(-1)).cuda(),
        router_bias=torch.from_numpy(synth.zipf_bias(SEED)).cuda() if zipf else None).prepare(ctx)


def _rank(rank, world, port, outdir, zipf, native):
    import torch
    import torch.distributed as dist
    from willow_v2_b200 import moe
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = moe.Context(rank)
        per = 256 // world
        store = moe.ExpertStore(1, ctx=ctx, expert_range=(rank * per, (rank + 1) * per))
        store.fill_synthetic(SEED)
        lw = _weights(moe, torch, ctx, zipf)
        x = torch.from_numpy(synth.hidden(SEED, TOKENS_PER_RANK * world, step=33)).to(torch.bfloat16)
        mine = x[rank * TOKENS_PER_RANK:(rank + 1) * TOKENS_PER_RANK].cuda()
        if native:
            from willow_v2_b200.lib import lib
            moe.ep_init(ctx)
            outs = []
            for chunks in (4, 1, 3):  # the result does not depend on the chunking
                lib.wmoe_ep_set_chunks(ctx.handle, chunks)
                outs.append(moe.moe_forward_ep_native(store, LAYER, mine, lw, out_dtype=torch.float32))
            # a rank with no tokens still takes part in every exchange
            empty = moe.moe_forward_ep_native(store, LAYER, mine[:0], lw, out_dtype=torch.float32) if rank == 1 \
                else moe.moe_forward_ep_native(store, LAYER, mine, lw, out_dtype=torch.float32)
            assert empty.shape[0] == (0 if rank == 1 else TOKENS_PER_RANK)
        else:
            outs = [moe.moe_forward_ep(store, LAYER, mine, lw, out_dtype=torch.float32) for _ in range(2)]
        torch.cuda.synchronize()
        ctx.check_device()
        if native:
            ctx.ep_finalize()
        assert all(torch.equal(outs[0], o) for o in outs[1:])
        np.save(os.path.join(outdir, f"out{rank}.npy"), outs[0].cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("zipf,native", [(False, False), (True, False), (False, True), (True, True)])
def test_ep_over_nccl_matches_single_gpu(zipf, native):
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(world, _free_port(), d, zipf, native), nprocs=world, start_method="spawn")
        outs = [np.load(os.path.join(d, f"out{r}.npy")) for r in range(world)]
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import lib
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    full = moe.ExpertStore(1, ctx=ctx)
    full.fill_synthetic(SEED)
    lw = _weights(moe, torch, ctx, zipf)
    x = torch.from_numpy(synth.hidden(SEED, TOKENS_PER_RANK * world, step=33)).to(torch.bfloat16).cuda()
    prev = lib.wmoe_set_prefill_threshold(ctx.handle, 1)
    try:
        ref = moe.moe_forward(full, LAYER, x, lw, out_dtype=torch.float32).cpu().numpy()
    finally:
        lib.wmoe_set_prefill_threshold(ctx.handle, prev)
    for r in range(world):
        assert np.array_equal(outs[r], ref[r * TOKENS_PER_RANK:(r + 1) * TOKENS_PER_RANK]), r


@pytest.mark.parametrize("zipf", [False, True])
def test_ep_native_one_rank_matches_single_gpu(zipf):
    """The library's own EP path on a one-rank communicator (one GPU): the count all-gather, the exchange window,
    the copy-engine copies and the barriers all run; the output equals the single-GPU layer bit for bit for every
    chunk count."""
    import torch
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(1, _free_port(), d, zipf, True), nprocs=1, start_method="spawn")
        out = np.load(os.path.join(d, "out0.npy"))
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import lib
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    full = moe.ExpertStore(1, ctx=ctx)
    full.fill_synthetic(SEED)
    lw = _weights(moe, torch, ctx, zipf)
    x = torch.from_numpy(synth.hidden(SEED, TOKENS_PER_RANK, step=33)).to(torch.bfloat16).cuda()
    prev = lib.wmoe_set_prefill_threshold(ctx.handle, 1)
    try:
        ref = moe.moe_forward(full, LAYER, x, lw, out_dtype=torch.float32).cpu().numpy()
    finally:
        lib.wmoe_set_prefill_threshold(ctx.handle, prev)
    assert np.array_equal(out, ref)


STACK_LAYERS, STACK_TOKENS = 3, 512


def _stack_weights(moe, torch, ctx):
    return [moe.LayerWeights(
        router_w=torch.from_numpy(synth.router_weight(SEED, l)).cuda(),
        shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, l)).cuda(),
        shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, l, 256).reshape(-1)).cuda(),
        shared_down=torch.from_numpy(synth.expert_down(SEED, l, 256).reshape(-1)).cuda(),
        router_bias=torch.from_numpy(synth.zipf_bias(SEED + l)).cuda()).prepare(ctx) for l in range(STACK_LAYERS)]


def _stack_rank(rank, world, port, outdir):
    """wmoe_prefill_stack after wmoe_ep_init: every layer over the library's communicator, the residual epilogue in
    each chunk's combine."""
    import torch
    import torch.distributed as dist
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import lib
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = moe.Context(rank)
        per = 256 // world
        store = moe.ExpertStore(STACK_LAYERS, ctx=ctx, expert_range=(rank * per, (rank + 1) * per))
        store.fill_synthetic(SEED)
        lws = _stack_weights(moe, torch, ctx)
        h = torch.from_numpy(synth.hidden(SEED, STACK_TOKENS * world, step=77)[rank * STACK_TOKENS:
                                                                                (rank + 1) * STACK_TOKENS]).cuda()
        moe.ep_init(ctx)
        outs = []
        for chunks in (1, 2):  # the result does not depend on the chunking
            lib.wmoe_ep_set_chunks(ctx.handle, chunks)
            outs.append(moe.prefill_stack(store, lws, h))
        # a rank without tokens still takes part in every layer's exchanges; the other ranks' rows do not change
        part = moe.prefill_stack(store, lws, h[:0] if rank == world - 1 and world > 1 else h)
        torch.cuda.synchronize()
        ctx.check_device()
        ctx.ep_finalize()
        assert torch.equal(outs[0], outs[1])
        assert part.shape[0] == 0 if rank == world - 1 and world > 1 else torch.equal(part, outs[0])
        np.save(os.path.join(outdir, f"stack{rank}.npy"), outs[0].cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _stack_reference(world):
    import torch
    from willow_v2_b200 import moe
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    full = moe.ExpertStore(STACK_LAYERS, ctx=ctx)
    full.fill_synthetic(SEED)
    h = torch.from_numpy(synth.hidden(SEED, STACK_TOKENS * world, step=77)).cuda()
    out = moe.prefill_stack(full, _stack_weights(moe, torch, ctx), h).cpu().numpy()
    full.close()
    return out


def test_ep_prefill_stack_one_rank_matches_single_gpu():
    """The stack over a one-rank communicator (one GPU) gives the single-GPU stack bit for bit."""
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_stack_rank, args=(1, _free_port(), d), nprocs=1, start_method="spawn")
        out = np.load(os.path.join(d, "stack0.npy"))
    assert np.array_equal(out, _stack_reference(1))


def test_ep_prefill_stack_matches_single_gpu():
    """Three layers of Zipf-routed tokens through wmoe_prefill_stack on 2, 4 or 8 ranks: every rank's rows equal the
    single-GPU stack's bit for bit."""
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_stack_rank, args=(world, _free_port(), d), nprocs=world, start_method="spawn")
        outs = [np.load(os.path.join(d, f"stack{r}.npy")) for r in range(world)]
    ref = _stack_reference(world)
    for r in range(world):
        assert np.array_equal(outs[r], ref[r * STACK_TOKENS:(r + 1) * STACK_TOKENS]), r


def _mismatch_rank(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import WmoeError, lib
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = moe.Context(rank)
        per = 256 // world
        store = moe.ExpertStore(1, ctx=ctx, expert_range=(rank * per, (rank + 1) * per))
        store.fill_synthetic(SEED)
        lw = _weights(moe, torch, ctx, False)
        x = torch.from_numpy(synth.hidden(SEED, 256, step=44)).to(torch.bfloat16).cuda()
        moe.ep_init(ctx)
        lib.wmoe_ep_set_chunks(ctx.handle, 1 + rank % 2)  # ranks disagree
        try:
            moe.moe_forward_ep_native(store, LAYER, x, lw)
            raised = False
        except WmoeError as e:
            raised = "chunk counts" in str(e)
        lib.wmoe_ep_set_chunks(ctx.handle, 2)  # agree again: the communicator is still usable
        out = moe.moe_forward_ep_native(store, LAYER, x, lw)
        torch.cuda.synchronize()
        ctx.ep_finalize()
        np.save(os.path.join(outdir, f"ok{rank}.npy"), np.array([raised, bool(torch.isfinite(out.float()).all())]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ep_chunk_mismatch_is_an_error_on_every_rank():
    """Ranks configured with different chunk counts get WMOE_ERR_INVALID from the same call (the fixed-size count
    exchange carries the count) instead of mismatched exchanges; the next agreeing call works."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_mismatch_rank, args=(2, _free_port(), d), nprocs=2, start_method="spawn")
        for r in range(2):
            raised, finite = np.load(os.path.join(d, f"ok{r}.npy"))
            assert raised and finite, r


def _leave_rank(rank, world, port, outdir):
    """Two ranks take one step together; rank 1 then leaves between steps (nothing of it in flight) and exits; rank
    0's next layer must come back with WMOE_ERR_NCCL within the context's timeout, and its GPU stays usable."""
    import time
    import torch
    import torch.distributed as dist
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import ERR_NCCL, WmoeError
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # plain peer transfers: nothing of a leaving rank bound to a multicast object
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # the test's own coordination over gloo, so that the survivor's teardown does not wait on the rank that left
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    ctx = moe.Context(rank)
    per = 256 // world
    store = moe.ExpertStore(1, ctx=ctx, expert_range=(rank * per, (rank + 1) * per))
    store.fill_synthetic(SEED)
    lw = _weights(moe, torch, ctx, False)
    x = torch.from_numpy(synth.hidden(SEED, 512, step=55 + rank)).to(torch.bfloat16).cuda()
    moe.ep_init(ctx)
    ctx.ep_set_timeout(3000)
    first = moe.moe_forward_ep_native(store, LAYER, x, lw)
    torch.cuda.synchronize()
    dist.barrier()
    ready = os.path.join(outdir, "rank0_out_of_barrier")
    if rank == 1:
        torch.cuda.synchronize()  # nothing of it in flight
        while not os.path.exists(ready):  # rank 0 is past the barrier: only its next layer sees this rank gone
            time.sleep(0.05)
        np.save(os.path.join(outdir, "left1.npy"), np.array([1.0]))
        os._exit(0)  # leaves without a goodbye (no finalize, no destroy), as a failed rank would
    open(ready, "w").close()
    time.sleep(1.0)

    def say(what):
        print(f"rank 0: {what} at {time.time() - t0:.2f} s", flush=True)

    t0 = time.time()
    code = 0
    try:
        moe.moe_forward_ep_native(store, LAYER, x, lw)
        say("call returned")
        torch.cuda.synchronize()
    except WmoeError as e:
        code = e.code
        say(f"error {e}")
    waited = time.time() - t0
    # the communicator is gone, the GPU is not: a single-GPU layer still runs, with a clean device status
    ctx.ep_finalize()
    say("finalized")
    full = moe.ExpertStore(1, ctx=ctx)
    full.fill_synthetic(SEED)
    again = moe.moe_forward(full, LAYER, x, lw)
    torch.cuda.synchronize()
    ok = bool(torch.isfinite(again.float()).all()) and bool(torch.isfinite(first.float()).all())
    ok = ok and ctx.device_status() == 0
    say("single-GPU layer ran")
    np.save(os.path.join(outdir, "left0.npy"), np.array([float(code == ERR_NCCL), waited, float(ok)]))
    os._exit(0)


def test_ep_rank_leaving_is_an_nccl_error():
    """A rank that leaves between steps: the survivor's next wmoe_moe_forward_ep returns WMOE_ERR_NCCL within its
    3 s timeout (the count exchange's bounded wait aborts the communicator) instead of hanging; no GPU is faulted
    or left waiting."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    with tempfile.TemporaryDirectory() as d:
        ctxs = mp.start_processes(_leave_rank, args=(2, _free_port(), d), nprocs=2, start_method="spawn", join=False)
        deadline = time.time() + 120
        while not ctxs.join(timeout=max(1.0, deadline - time.time())) and time.time() < deadline:
            pass
        for p in ctxs.processes:  # a rank still running at the deadline is a failure; it must not outlive the test
            if p.is_alive():
                p.kill()
        assert os.path.exists(os.path.join(d, "left1.npy"))
        nccl_error, waited, ok = np.load(os.path.join(d, "left0.npy"))
        assert nccl_error == 1.0 and ok == 1.0
        assert waited < 20.0, waited
