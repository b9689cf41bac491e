"""The expert-parallel dispatch kernels on one GPU, through the C ABI: lk_moe_rank_plan against a stable numpy sort
of the assignments by destination rank (order, pos and counts, exactly), and lk_moe_gather_rows against indexing
(bit for bit). The sorted rows combined through pos equal the combine of the rows in assignment order."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import ops as _ops
    return _ops


@pytest.mark.parametrize("tokens,ku,E,world", [(1, 8, 128, 8), (37, 4, 32, 4), (4096, 8, 128, 8), (500, 2, 64, 2),
                                               (3, 8, 256, 32), (8192, 8, 128, 1)])
def test_rank_plan_and_gather(ops, tokens, ku, E, world):
    rng = np.random.default_rng(tokens + world)
    ids = np.stack([rng.permutation(E)[:ku] for _ in range(tokens)]).astype(np.int32)
    n_local = E // world
    order, pos, counts = ops.moe_rank_plan(torch.from_numpy(ids).cuda(), n_local, world)
    dest = ids.reshape(-1) // n_local
    ref_order = np.argsort(dest, kind="stable")
    ref_pos = np.empty_like(ref_order)
    ref_pos[ref_order] = np.arange(ref_order.size)
    assert np.array_equal(order.cpu().numpy(), ref_order)
    assert np.array_equal(pos.cpu().numpy(), ref_pos)
    assert np.array_equal(counts.cpu().numpy(), np.bincount(dest, minlength=world))
    for dt in (torch.float32, torch.bfloat16):
        x = torch.randn(tokens, 2048, device="cuda").to(dt)
        rows, eid = ops.moe_gather_rows(order, torch.from_numpy(ids).cuda(), x, ku, n_local)
        assert torch.equal(rows, x.index_select(0, order.long() // ku))
        assert np.array_equal(eid.cpu().numpy(), ids.reshape(-1)[ref_order] % n_local)
    ys = torch.randn(tokens * ku, 256, device="cuda")
    wts = torch.rand(tokens, ku, device="cuda")
    sorted_ys = ys.index_select(0, order.long())
    y1 = ops.moe_combine_sorted(sorted_ys, pos.view(tokens, ku), wts)
    y2 = ops.moe_combine(ys, wts)
    assert torch.equal(y1, y2)
    assert ops.device_status() == 0
