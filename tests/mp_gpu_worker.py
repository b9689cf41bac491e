"""One rank of the multi-GPU parity check (launched by test_gpu_multi.py under torchrun, one process per GPU).

Checks, on every rank:
  * ShardedGemm ('p2p': all-gather fused into the GEMM epilogue over NVLink; 'collective': NCCL all-gather) equals
    the single-GPU GEMM of the full weight (the same tiles' arithmetic: relative L2 <= 1e-6), in store and swiglu
    modes, on four calls in a row with different activations (the two peer buffers each used twice); every result is
    kept -- as the copy `out=` makes for 'p2p', whose own result lives until the next call -- and all are compared
    after the last call;
  * ExpertParallelMoE (experts sharded, tokens exchanged by NCCL all_to_all) against the oracle's float64 expert FFN
    within 1e-3, for a prefill-sized and a decode-sized token count.
Exits non-zero on a mismatch."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from loom_skills_b200 import ops  # noqa: E402
from loom_skills_b200.parallel import ExpertParallelMoE, ShardedGemm, shard_range  # noqa: E402
from oracle import qmm_oracle as O  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    failures = []
    rng = np.random.default_rng(7)
    # ---------------------------------------------------------------- sharded GEMM
    n, k, rows = 1024 * world, 1024, 300
    w = O.quantize_iq4_nl((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    w2 = O.quantize_iq4_nl((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = torch.from_numpy(rng.standard_normal((rows, k)).astype(np.float32)).cuda().to(torch.bfloat16)
    x16, sc = ops.row_scale_f16(x)
    wd, w2d = torch.from_numpy(w).cuda(), torch.from_numpy(w2).cuda()
    c0, c1 = shard_range(n, world, rank)
    xs = [ops.row_scale_f16((x.float() * (1.0 + 0.5 * c)).to(torch.bfloat16)) for c in range(4)]
    for mode in ("store", "swiglu"):
        fulls = [ops.gemm("iq4_nl", mode, a16, asc, wd, n, w2=w2d if mode == "swiglu" else None) for a16, asc in xs]
        for exchange in ("p2p", "collective"):
            sg = ShardedGemm("iq4_nl", mode, wd[c0:c1].contiguous(), n, k, exchange=exchange,
                             w2_local=w2d[c0:c1].contiguous() if mode == "swiglu" else None)
            kept = []
            for a16, asc in xs:
                if exchange == "p2p":
                    kept.append(sg(a16, asc, out=torch.empty(rows, n, device="cuda")))
                else:
                    kept.append(sg(a16, asc))
            torch.cuda.synchronize()
            for call, (y, full) in enumerate(zip(kept, fulls)):
                err = float((y - full).norm() / full.norm())
                if not err <= 1e-6:
                    failures.append(f"sharded {mode} {exchange} call {call}: rel {err}")
            dist.barrier()
            sg.close()
    # ---------------------------------------------------------------- expert-parallel MoE
    E, ku, h, f = 4 * world, 2, 256, 256
    w_gu = O.quantize_q4_0((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
    w_dn = O.quantize_q4_0((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32))
    nl = E // world
    moe = ExpertParallelMoE("q4_0", torch.from_numpy(w_gu[rank * nl * 2 * f:(rank + 1) * nl * 2 * f]).cuda(),
                            torch.from_numpy(w_dn[rank * nl * h:(rank + 1) * nl * h]).cuda(), h, f, E, ku)
    for t in (200, 3):
        trng = np.random.default_rng(1000 * t + rank)
        xt = trng.standard_normal((t, h)).astype(np.float32)
        logits = trng.standard_normal((t, E)).astype(np.float32)
        y = moe(torch.from_numpy(xt).cuda(), torch.from_numpy(logits).cuda()).cpu().numpy()
        ids, wts = O.route_ref(logits, ku)
        ref = O.moe_ffn_ref(xt, ids, wts, w_gu.reshape(E, 2 * f, -1), w_dn.reshape(E, h, -1), "q4_0", h, f, E)
        err = O.rel_l2(y, ref)
        if not err <= 1e-3:
            failures.append(f"expert-parallel MoE t={t}: rel {err}")
    status = ops.device_status()
    if status:
        failures.append(f"device status {status}")
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: {'OK' if not failures else failures}", flush=True)
    sys.exit(1 if failures else 0)


if __name__ == "__main__":
    main()
