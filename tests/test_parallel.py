"""Host logic of the multi-GPU forms on CPU ranks (gloo, world size 2) with the oracle as the compute:
shard ranges, the column all-gather of ShardedGemm, and the dispatch / exchange / return / combine of
ExpertParallelMoE. The GPU forms (P2P epilogue stores, NCCL) are covered by test_gpu_multi.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from loom_skills_b200.parallel import ExpertParallelMoE, ShardedGemm, shard_range
from oracle import qmm_oracle as O


def test_shard_range_covers_and_aligns():
    for n in (16, 4096, 5120, 27648, 27648 + 48):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(c0 % 16 == 0 and c1 % 16 == 0 for c0, c1 in spans)
            widths = [c1 - c0 for c0, c1 in spans]
            assert max(widths) - min(widths) <= 16
    with pytest.raises(ValueError):
        shard_range(100, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_gemm(fmt, mode, x16, scales, w, n, w2=None):
    k = x16.shape[1]
    y = O.gemm_ref(fmt, w.numpy(), x16.numpy(), scales.numpy(), n, k, mode=mode,
                   w2=None if w2 is None else w2.numpy())
    return torch.from_numpy(y.astype(np.float32))


class OracleMoE:
    """ExpertParallelMoE's compute steps restated on the CPU (float64 dequant + products)."""

    def __init__(self, fmt):
        self.fmt = fmt

    def route(self, logits, n_experts, ku):
        ids, wts = O.route_ref(logits.numpy(), ku)
        return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(wts.astype(np.float32))

    def experts(self, x, eids, w_gu, w_dn, h, f, n_local):
        out = np.zeros((x.shape[0], h), np.float64)
        xs = x.double().numpy()
        for e in np.unique(eids.numpy()):
            sel = np.nonzero(eids.numpy() == e)[0]
            rb_h, rb_f = w_gu.shape[1], w_dn.shape[1]
            gu = O.dequant(self.fmt, w_gu[e * 2 * f:(e + 1) * 2 * f].numpy(), h).reshape(2 * f, h)
            dn = O.dequant(self.fmt, w_dn[e * h:(e + 1) * h].numpy(), f).reshape(h, f)
            pair = xs[sel] @ gu.T.astype(np.float64)
            act = O.silu(pair[:, :f]) * pair[:, f:]
            out[sel] = act @ dn.T.astype(np.float64)
        return torch.from_numpy(out.astype(np.float32))

    def plan(self, ids, n_local, world):
        dest = (ids.reshape(-1) // n_local).long()
        order = torch.argsort(dest, stable=True)
        pos = torch.empty_like(order)
        pos[order] = torch.arange(order.numel())
        return order.to(torch.int32), pos.to(torch.int32), torch.bincount(dest, minlength=world).to(torch.int32)

    def gather(self, order, ids, x, ku, n_local):
        o = order.long()
        return x.index_select(0, o // ku).contiguous(), (ids.reshape(-1).long()[o] % n_local).to(torch.int32)

    def combine_sorted(self, ys, pos, wts):
        t, ku = wts.shape
        return (ys[pos.long()].view(t, ku, -1).double() * wts.double()[:, :, None]).sum(1).float()


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(5)
        # ---- sharded GEMM: IQ4_NL weights, replicated activations
        n, k, rows = 96, 256, 7
        w = O.quantize_iq4_nl((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        x = rng.standard_normal((rows, k)).astype(np.float32)
        _, x16, sc = (None, *O.row_scale_f16(x))
        c0, c1 = shard_range(n, world, rank)
        sg = ShardedGemm("iq4_nl", "store", torch.from_numpy(w[c0:c1]), n, k, exchange="collective",
                         gemm_fn=oracle_gemm)
        y = sg(torch.from_numpy(x16), torch.from_numpy(sc)).numpy()
        ref = O.gemm_ref("iq4_nl", w, x16, sc, n, k)
        gemm_err = O.rel_l2(y, ref)
        # ---- expert-parallel MoE: Q4_0 experts, each rank its own tokens
        E, ku, h, f = 4, 2, 64, 32
        w_gu = O.quantize_q4_0((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
        w_dn = O.quantize_q4_0((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32))
        trng = np.random.default_rng(100 + rank)
        t = 5 + 3 * rank
        xt = trng.standard_normal((t, h)).astype(np.float32)
        logits = trng.standard_normal((t, E)).astype(np.float32)
        nl = E // world
        moe = ExpertParallelMoE("q4_0", torch.from_numpy(w_gu[rank * nl * 2 * f:(rank + 1) * nl * 2 * f]),
                                torch.from_numpy(w_dn[rank * nl * h:(rank + 1) * nl * h]), h, f, E, ku,
                                backend=OracleMoE("q4_0"))
        ym = moe(torch.from_numpy(xt), torch.from_numpy(logits)).numpy()
        ids, wts = O.route_ref(logits, ku)
        mref = O.moe_ffn_ref(xt, ids, wts, w_gu.reshape(E, 2 * f, -1), w_dn.reshape(E, h, -1), "q4_0", h, f, E)
        q.put((rank, gemm_err, O.rel_l2(ym, mref)))
        dist.destroy_process_group()
    except Exception as e:   # report instead of hanging the parent
        q.put((rank, repr(e), None))


def test_two_ranks_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, gerr, merr in results:
        assert not isinstance(gerr, str), gerr
        assert gerr < 1e-6, (rank, gerr)
        assert merr < 1e-6, (rank, merr)
