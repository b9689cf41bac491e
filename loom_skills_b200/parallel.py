"""Multi-GPU forms of the quantized-matmul path: one process per GPU, torch.distributed for the plumbing.

The reference runs on one device and has no collectives (its workgroup reductions are on-chip); the two sharded forms
here are the ones asked of this build for the GPUs of one NVSwitch box:

ShardedGemm   N-sharded prefill GEMM. Rank r owns output columns [c0_r, c1_r) -- its slice of the packed weight rows
              -- and the full y [rows][n] is all-gathered:
                'p2p'        lk_gemm_allgather stores every finished output tile into every rank's y buffer over
                             NVLink (the all-gather fused into the GEMM epilogue), then the ranks meet at a barrier.
                             y buffers are cudaMalloc'd and shared by interprocess handles (lk_peer_*), two of them
                             used in turn so one barrier per call orders writers against readers.
                'collective' local GEMM into [rows][n_r], all_gather_into_tensor (NCCL; gloo on the CPU), then the
                             rank-major blocks are interleaved into columns.
ExpertParallelMoE  experts sharded over ranks (rank r owns experts [r*E/N, (r+1)*E/N)). Each rank routes its own
              tokens, sends every assignment's token row to the rank owning its expert (all_to_all_single, counts
              first), runs the owned experts over the rows it received (the bucketed grouped-GEMM pipeline with one
              assignment per row), sends the results back the same way and combines with its routing weights.

The compute steps are injectable (`gemm_fn`, `backend`) so the host logic -- shard ranges, exchanges, permutations --
is tested on CPU ranks over gloo with the oracle as the compute; on GPUs they are liblk's kernels.
"""
import ctypes

import torch
import torch.distributed as dist

ALIGN = 16   # output columns per shard are a multiple of this (the GEMM's n % 16 contract)


def shard_range(n, world, rank, align=ALIGN):
    """[c0, c1) of rank's share of n columns: contiguous, multiples of `align`, sizes differing by at most `align`."""
    if n % align:
        raise ValueError(f"n={n} is not a multiple of {align}")
    units = n // align
    base, extra = divmod(units, world)
    c0 = (rank * base + min(rank, extra)) * align
    c1 = c0 + (base + (1 if rank < extra else 0)) * align
    return c0, c1


def _world(group):
    """(world size, rank) of `group`; a process without a process group is a world of one."""
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


# ------------------------------------------------------------------------------------------------------------------
# peer buffers (CUDA interprocess handles)
# ------------------------------------------------------------------------------------------------------------------
class _DevArray:
    """A raw device pointer as a torch tensor view (CUDA array interface, no copy)."""

    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffers:
    """One [rows][n] f32 buffer per rank, every rank holding device pointers to all of them (its own first)."""

    def __init__(self, rows, n, group=None):
        from . import _lib as L
        self.L = L.load()
        self.world, self.rank = _world(group)
        self.shape = (rows, n)
        nbytes = rows * n * 4
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        L.check(self.L.lk_peer_alloc(nbytes, ctypes.byref(own), handle), "lk_peer_alloc")
        self.own = own.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                continue
            p = ctypes.c_void_p()
            L.check(self.L.lk_peer_open((ctypes.c_uint8 * 64).from_buffer_copy(handles[r]), ctypes.byref(p)),
                    "lk_peer_open")
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.ptrs = [self.own] + ptrs
        self.dst = (ctypes.c_void_p * len(self.ptrs))(*self.ptrs)
        self.tensor = torch.as_tensor(_DevArray(self.own, self.shape), device="cuda")

    def close(self):
        for p in self.opened:
            self.L.lk_peer_close(p)
        self.opened = []
        if self.own:
            self.L.lk_peer_free(self.own)
            self.own = None


# ------------------------------------------------------------------------------------------------------------------
# N-sharded GEMM
# ------------------------------------------------------------------------------------------------------------------
class ShardedGemm:
    """y [rows][n] = GEMM(x16, scales, W) with W's rows (output columns) sharded over the ranks of `group`.

    w_local: this rank's packed weight rows [c1 - c0][row_bytes] (shard_range(n, world, rank)); w2_local: its up
    rows for mode 'swiglu'. Every rank passes the same x16/scales (replicated activations).

    Lifetime of the result: the 'collective' exchange returns a new tensor. The 'p2p' exchange returns a view of one
    of two peer buffers that the ranks write in turn: it stays valid until this rank's next call on this object
    (after that call the peers may already be writing the buffer for the call after). Pass `out` to have the
    gathered result copied into a tensor of your own instead (on the current stream, before the call returns)."""

    def __init__(self, fmt, mode, w_local, n, k, group=None, exchange="p2p", w2_local=None, gemm_fn=None):
        self.fmt, self.mode, self.n, self.k, self.group = fmt, mode, n, k, group
        self.world, self.rank = _world(group)
        self.c0, self.c1 = shard_range(n, self.world, self.rank)
        self.w, self.w2 = w_local, w2_local
        self.exchange = exchange
        self.gemm_fn = gemm_fn
        self._bufs = {}
        self._turn = 0
        self._flag = None

    def _barrier(self, device):
        if self.world == 1:
            return
        if self._flag is None:
            self._flag = torch.zeros(1, device=device)
        dist.all_reduce(self._flag, group=self.group)

    def __call__(self, x16, scales, out=None):
        rows = x16.shape[0]
        y = self._p2p(x16, scales, rows) if self.exchange == "p2p" else self._collective(x16, scales, rows)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def _local(self, x16, scales):
        fn = self.gemm_fn
        if fn is None:
            from . import ops
            fn = ops.gemm
        return fn(self.fmt, self.mode, x16, scales, self.w, self.c1 - self.c0, w2=self.w2)

    def _collective(self, x16, scales, rows):
        y_local = self._local(x16, scales).contiguous()
        if self.world == 1:
            return y_local
        widths = [shard_range(self.n, self.world, r) for r in range(self.world)]
        if all(c1 - c0 == widths[0][1] - widths[0][0] for c0, c1 in widths):
            buf = torch.empty(self.world * rows, y_local.shape[1], dtype=y_local.dtype, device=y_local.device)
            dist.all_gather_into_tensor(buf, y_local, group=self.group)
            return buf.view(self.world, rows, -1).permute(1, 0, 2).reshape(rows, self.n)
        parts = [torch.empty(rows, c1 - c0, dtype=y_local.dtype, device=y_local.device) for c0, c1 in widths]
        dist.all_gather(parts, y_local, group=self.group)
        return torch.cat(parts, 1)

    def _p2p(self, x16, scales, rows):
        from . import _lib as L
        key = rows
        if key not in self._bufs:
            self._bufs[key] = [PeerBuffers(rows, self.n, self.group) for _ in range(2)]
        buf = self._bufs[key][self._turn]
        self._turn ^= 1
        lib = L.load()
        m = L.MODE_IDS[self.mode]
        L.check(lib.lk_gemm_allgather(L.FMT_IDS[self.fmt], m, rows, self.k, self.c1 - self.c0, x16.data_ptr(),
                                      scales.data_ptr(), self.w.data_ptr(),
                                      None if self.w2 is None else self.w2.data_ptr(), buf.dst, len(buf.ptrs), self.n,
                                      self.c0, torch.cuda.current_stream().cuda_stream), "lk_gemm_allgather")
        self._barrier(x16.device)   # every rank's tiles are in every buffer
        return buf.tensor

    def close(self):
        for pair in self._bufs.values():
            for b in pair:
                b.close()
        self._bufs = {}


# ------------------------------------------------------------------------------------------------------------------
# expert-parallel MoE
# ------------------------------------------------------------------------------------------------------------------
class GpuMoEBackend:
    """The compute steps of ExpertParallelMoE on liblk's kernels."""

    def __init__(self, fmt):
        self.fmt = fmt

    def route(self, logits, n_experts, ku):
        from . import ops
        return ops.moe_route(logits, n_experts, ku)

    def plan(self, ids, n_local, world):
        """-> (order, pos, counts): the assignments stably sorted by destination rank (lk_moe_rank_plan)."""
        from . import ops
        return ops.moe_rank_plan(ids, n_local, world)

    def gather(self, order, ids, x, ku, n_local):
        """-> (send rows x[order // ku], their local expert ids) (lk_moe_gather_rows)."""
        from . import ops
        return ops.moe_gather_rows(order, ids, x, ku, n_local)

    def experts(self, x, eids, w_gu, w_dn, h, f, n_local):
        """rows x [R][h], each with one local expert eids[R] -> Wd[e] (silu(Wg[e] x) * (Wu[e] x)) [R][h]."""
        from . import ops
        r = x.shape[0]
        if r == 0:
            return torch.zeros(0, h, dtype=torch.float32, device=x.device)
        # decode-sized: per-row expert matvecs (the crossover ops.moe_ffn measured; grouped by expert up to 1024 rows)
        if r < 192 or (r <= 1024 and ops._grouped_decode(self.fmt, None, x.dtype, h, f, n_local)):
            act = ops.moe_expert_mv(self.fmt, "gu", eids, x, w_gu, f, h, 1, n_local, fused=True)
            return ops.moe_expert_mv(self.fmt, "dn", eids, act, w_dn, h, f, 1, n_local)
        ti, rm, pos = ops.moe_bucket(eids.view(r, 1), n_local)
        x16, sc = ops.moe_row_scale_gather(x, rm, 1)   # the rows in bucket order: gate/up reads plain tiles
        act = ops.moe_grouped_gemm(self.fmt, "swiglu_sorted", ti, rm, x16, sc, w_gu, f, 1, n_local, fused=True)
        a16, asc = ops.row_scale_f16(act)
        ys = ops.moe_grouped_gemm(self.fmt, "store", ti, rm, a16, asc, w_dn, h, 1, n_local)
        ones = torch.ones(r, 1, dtype=torch.float32, device=x.device)
        return ops.moe_combine_sorted(ys, pos, ones)

    def combine_sorted(self, ys, pos, wts):
        """y[t] = sum_k wts[t,k] ys[pos[t,k]] in k order (lk_moe_combine_sorted)."""
        from . import ops
        return ops.moe_combine_sorted(ys, pos.view(wts.shape), wts)


class ExpertParallelMoE:
    """The routed expert FFN with experts sharded over the ranks of `group` (E % world == 0).

    w_gu_local: packed rows of this rank's experts, 2f rows each (gate then up) of h values; w_dn_local: h rows each
    of f values. Each rank passes its own tokens. The dispatch runs on the GPU: the routing, a stable sort of the
    assignments by destination rank, the gather of the send rows, and the weighted combine of the returned rows in
    that order; NCCL moves the counts and the rows. The counts cross to the host once per call, as NCCL's variable
    all-to-all takes its split sizes there."""

    def __init__(self, fmt, w_gu_local, w_dn_local, h, f, n_experts, ku, group=None, backend=None):
        self.world, self.rank = _world(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        self.n_local = n_experts // self.world
        self.h, self.f, self.E, self.ku, self.group = h, f, n_experts, ku, group
        self.w_gu, self.w_dn = w_gu_local, w_dn_local
        self.be = backend if backend is not None else GpuMoEBackend(fmt)
        self.times = None   # per-stage device times of the last call when timed (ms), see __call__

    def __call__(self, x, logits, timed=False):
        t = x.shape[0]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if timed else None
        mark = (lambda i: ev[i].record()) if timed else (lambda i: None)
        mark(0)
        ids, wts = self.be.route(logits, self.E, self.ku)
        order, pos, send_counts = self.be.plan(ids, self.n_local, self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_x, send_e = self.be.gather(order, ids, x, self.ku, self.n_local)
        counts = torch.cat([send_counts, recv_counts]).tolist()   # the split sizes NCCL takes on the host
        sc, rc = counts[:self.world], counts[self.world:]
        recv_x = torch.empty(sum(rc), self.h, dtype=x.dtype, device=x.device)
        recv_e = torch.empty(sum(rc), dtype=torch.int32, device=x.device)
        mark(1)
        dist.all_to_all_single(recv_x, send_x, rc, sc, group=self.group)
        dist.all_to_all_single(recv_e, send_e, rc, sc, group=self.group)
        mark(2)
        ys_recv = self.be.experts(recv_x, recv_e, self.w_gu, self.w_dn, self.h, self.f, self.n_local).contiguous()
        mark(3)
        ys_back = torch.empty(t * self.ku, self.h, dtype=ys_recv.dtype, device=x.device)
        dist.all_to_all_single(ys_back, ys_recv, sc, rc, group=self.group)
        mark(4)
        y = self.be.combine_sorted(ys_back, pos, wts)
        if timed:
            torch.cuda.synchronize()
            self.times = {"route_plan_gather_ms": ev[0].elapsed_time(ev[1]), "dispatch_a2a_ms": ev[1].elapsed_time(ev[2]),
                          "experts_ms": ev[2].elapsed_time(ev[3]), "return_a2a_ms": ev[3].elapsed_time(ev[4])}
        return y
