"""The expert-parallel exchange logic of moe_forward_ep on two gloo ranks on the CPU: the three per-rank steps are
restated here with the oracle (route, per-destination send order, pair lists, expert FFNs, combine in ascending
expert id), and the real all_to_all_single exchanges of counts, rows, pair lists and result rows run between
processes. The ranks' combined outputs must equal the single-process oracle MoE block on all tokens. (The GPU
kernels of the same three steps are checked against single-GPU results in test_gpu_ep.py.)"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import moe_oracle as ora
from willow_v2_b200 import synth

SEED, LAYER, E, TOKENS, WORLD = 0, 0, 256, 12, 2


class OracleEPOps:
    """CPU restatement of the per-rank steps (test infrastructure: the checker, not the product)."""

    def __init__(self):
        self.router = synth.router_weight(SEED, LAYER)
        self.gate = synth.shared_gate_weight(SEED, LAYER)
        self.cache = {}

    def weights(self, e):
        if e not in self.cache:
            self.cache[e] = (ora.dequantize(synth.expert_gate_up(SEED, LAYER, e), "Q4_K", (1024, 2048)),
                             ora.dequantize(synth.expert_down(SEED, LAYER, e), "Q6_K", (2048, 512)))
        return self.cache[e]

    def ffn(self, e, rows):
        gu, dn = self.weights(e)
        return ora.expert_gate(rows @ gu.T) @ dn.T

    def route_plan(self, store, x, lw, world, top_k):
        from willow_v2_b200.moe import EPPlan
        xn = x.numpy().astype(np.float32)
        T = xn.shape[0]
        w, sel = ora.route(xn @ self.router.T, top_k)
        shared_s = ora.sigmoid(xn @ self.gate)
        per = E // world
        rows, pairs, ret = [], [], np.zeros((T, top_k), dtype=np.int32)
        counts = np.zeros((2, world), dtype=np.int32)
        for d in range(world):
            toks = [t for t in range(T) if any(int(e) // per == d for e in sel[t])]
            counts[0, d] = len(toks)
            for local, t in enumerate(toks):
                rows.append(xn[t])
                for j in range(top_k):
                    if int(sel[t, j]) // per == d:
                        ret[t, j] = len(pairs)
                        pairs.append((local, int(sel[t, j])))
                        counts[1, d] += 1
        return EPPlan(topk_w=torch.from_numpy(w), topk_idx=torch.from_numpy(sel.astype(np.int32)),
                      shared_s=torch.from_numpy(shared_s.astype(np.float32)), counts=torch.from_numpy(counts),
                      send_buf=torch.from_numpy(np.array(rows, dtype=np.float32).reshape(-1, xn.shape[1])),
                      pair_list=torch.from_numpy(np.array(pairs, dtype=np.int32).reshape(-1, 2)),
                      ret_index=torch.from_numpy(ret))

    def experts(self, store, layer, world, recv_rows, recv_pairs, recv_buf, recv_pair_list, x, lw):
        base = np.concatenate([[0], np.cumsum(recv_rows)])
        pb = np.concatenate([[0], np.cumsum(recv_pairs)])
        rows = recv_buf.numpy()
        ys = []
        for s in range(world):
            for q in range(pb[s], pb[s + 1]):
                local, e = recv_pair_list[q].tolist()
                assert store.expert_range[0] <= e < store.expert_range[1]
                ys.append(self.ffn(e, rows[base[s] + local][None])[0])
        shared = self.ffn_shared(x.numpy().astype(np.float32))
        y = np.concatenate([np.array(ys, dtype=np.float32).reshape(-1, rows.shape[1]), shared])
        return torch.from_numpy(y)

    def ffn_shared(self, xn):
        gu = ora.dequantize(synth.expert_gate_up(SEED, LAYER, 256), "Q4_K", (1024, 2048))
        dn = ora.dequantize(synth.expert_down(SEED, LAYER, 256), "Q6_K", (2048, 512))
        return ora.expert_gate(xn @ gu.T) @ dn.T

    def combine(self, store, plan, y_ret, y_shared, out_dtype):
        T, k = plan.topk_idx.shape
        out = np.zeros((T, y_shared.shape[1]), dtype=np.float32)
        yr = y_ret.numpy()
        for t in range(T):
            for j in np.argsort(plan.topk_idx[t].numpy(), kind="stable"):  # ascending expert id
                out[t] += plan.topk_w[t, j].item() * yr[plan.ret_index[t, j].item()]
            out[t] += plan.shared_s[t].item() * y_shared[t].numpy()
        return torch.from_numpy(out)


def _rank(rank, world, port, outdir):
    import types
    import torch.distributed as dist
    from willow_v2_b200.moe import moe_forward_ep
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        per = E // world
        store = types.SimpleNamespace(experts=E, expert_range=(rank * per, (rank + 1) * per))
        x = synth.hidden(SEED, TOKENS, step=7)
        mine = torch.from_numpy(np.array_split(x, world)[rank])
        out = moe_forward_ep(store, LAYER, mine, None, ops=OracleEPOps(), out_dtype=torch.float32)
        np.save(os.path.join(outdir, f"out{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_exchange_on_two_gloo_ranks():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(WORLD, _free_port(), d), nprocs=WORLD, start_method="spawn")
        out = np.concatenate([np.load(os.path.join(d, f"out{r}.npy")) for r in range(WORLD)])
    ops = OracleEPOps()
    x = synth.hidden(SEED, TOKENS, step=7)
    want = ora.moe(x, ops.router, ops.weights, ops.weights(256), ops.gate)[0]
    err = float(np.linalg.norm(out - want) / np.linalg.norm(want))
    assert err < 1e-5, err


def _leave_rank(rank, world, port, outdir):
    """One step together, then rank 1 leaves between steps; rank 0's next exchange must fail within the process
    group's short timeout instead of waiting for good."""
    import datetime
    import time
    import types
    import torch.distributed as dist
    from willow_v2_b200.moe import moe_forward_ep
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    per = E // world
    store = types.SimpleNamespace(experts=E, expert_range=(rank * per, (rank + 1) * per))
    mine = torch.from_numpy(np.array_split(synth.hidden(SEED, TOKENS, step=9), world)[rank])
    moe_forward_ep(store, LAYER, mine, None, ops=OracleEPOps(), out_dtype=torch.float32)
    dist.barrier()
    ready = os.path.join(outdir, "rank0_out_of_barrier")
    if rank == 1:  # leaves once rank 0 is past the barrier (so that only the next exchange sees it gone)
        while not os.path.exists(ready):
            time.sleep(0.05)
        os._exit(0)
    open(ready, "w").close()
    time.sleep(1.0)
    t0 = time.time()
    failed = False
    try:
        moe_forward_ep(store, LAYER, mine, None, ops=OracleEPOps(), out_dtype=torch.float32)
    except RuntimeError:
        failed = True
    np.save(os.path.join(outdir, "left.npy"), np.array([float(failed), time.time() - t0]))
    os._exit(0)


def test_ep_rank_leaving_fails_the_next_exchange():
    """The exchange logic when a rank leaves between steps, on gloo ranks: the survivor's next layer raises from its
    first exchange within the group's 3 s timeout."""
    import time
    with tempfile.TemporaryDirectory() as d:
        ctxs = mp.start_processes(_leave_rank, args=(WORLD, _free_port(), d), nprocs=WORLD, start_method="spawn",
                                  join=False)
        deadline = time.time() + 120
        while not ctxs.join(timeout=max(1.0, deadline - time.time())) and time.time() < deadline:
            pass
        for p in ctxs.processes:
            if p.is_alive():
                p.kill()
        failed, waited = np.load(os.path.join(d, "left.npy"))
    assert failed == 1.0 and waited < 30.0, (failed, waited)

