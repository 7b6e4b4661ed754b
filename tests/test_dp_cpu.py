"""Host-side logic of the data-parallel step: the bucket-sharded optimizer layout (every bucket
split into one chunk per rank, chunks covering the flat buffer exactly once, each chunk aligned
for the 16-byte vector loads of the cast and NVLS kernels) and the transport choice."""
import pytest
import torch


@pytest.mark.parametrize("world", [2, 4, 8])
def test_bucket_chunks_cover_flat_buffer(world, monkeypatch):
    from llmt.config import get_config
    from llmt.models.llama import build_model
    from llmt.models.native import FlatParams
    from llmt.parallel.dp import BucketShardedAdamW
    # the shadow cast is a CUDA kernel; the layout under test is host-side
    monkeypatch.setattr(FlatParams, "refresh_shadow", lambda self: self.shadow.copy_(self.master))
    cfg = get_config("tiny256")
    flat = FlatParams(build_model(cfg, 32, seed=0), "cpu", pad_to=world, bucket_pad=True)
    assert len(flat.buckets) == cfg.L + 1  # one per block, then the emb / norm_f / head group
    assert flat.buckets[0][0] == 0 and flat.buckets[-1][1] == flat.numel
    for (a, b), (c, _) in zip(flat.buckets, flat.buckets[1:]):
        assert b == c
    cover = torch.zeros(flat.numel, dtype=torch.int32)
    m_total = None
    for r in range(world):
        opt = BucketShardedAdamW(flat, r, world)
        assert len(opt.ranges) == len(flat.buckets)
        moff = 0
        for (blo, bhi), (lo, hi), mo in zip(flat.buckets, opt.ranges, opt.moffs):
            c = (bhi - blo) // world
            assert (lo, hi) == (blo + r * c, blo + (r + 1) * c)
            assert lo % 8 == 0 and (hi - lo) % 8 == 0  # 16-byte bf16 vectors, 32-byte fp32 pairs
            assert mo == moff
            moff += hi - lo
            cover[lo:hi] += 1
        assert opt.exp_avg.numel() == moff
        m_total = moff if m_total is None else m_total
        assert moff == m_total  # every rank holds the same amount of optimizer state
    assert bool((cover == 1).all())


def test_overlap_modes_use_bucket_buffers():
    from llmt.parallel.dp import DataParallel
    assert DataParallel(2, 0, mode="nvls-overlap").overlap
    assert DataParallel(2, 0, mode="fused-overlap").overlap
    assert not DataParallel(2, 0, mode="nvls").overlap
    assert not DataParallel(2, 0, mode="nccl").overlap


def test_auto_mode_without_multicast_is_nccl():
    from llmt.parallel.dp import pick_mode
    assert pick_mode("nccl", 0) == "nccl"
    assert pick_mode("nvls-overlap", 0) == "nvls-overlap"
    if not torch.cuda.is_available():
        assert pick_mode("auto", 0) == "nccl"


def test_auto_mode_resolves_in_data_parallel():
    from llmt.parallel.dp import DataParallel
    dp = DataParallel(2, 0, mode="auto")
    assert dp.requested == "auto"
    if not torch.cuda.is_available():
        assert dp.mode == "nccl"
