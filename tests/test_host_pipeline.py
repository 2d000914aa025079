"""The pipelined host path's split (irx_run_host_chunks), checked without a GPU: which runs are
cut into chunks so that copies in and out overlap, and into how many."""
import pytest

from irptx_b200 import kir_author as ka


@pytest.mark.parametrize("kir, shard, nshards, want", [
    (ka.softmax(8192, 4096), 0, 1, 4),                    # 64 MB in, 64 MB out: 32 MB chunks
    (ka.softmax(8192, 4096), 1, 2, 2),                    # half of it per shard
    (ka.softmax(32768, 8192), 0, 1, 16),                  # 1 GB: at most 16 chunks
    (ka.rmsnorm(4096, 4096, d="f32"), 0, 1, 4),           # the weight goes in once, whole
    (ka.pointwise_relu_mul_affine(1 << 24), 0, 1, 6),     # 128 MB in, 64 MB out
    (ka.matmul(4096, 4096, 4096), 0, 1, 3),               # A whole, B and C by columns
    (ka.attention(8, 16, 1024, 128, causal=True), 0, 1, 4),
], ids=["softmax", "softmax_shard", "softmax_config", "rmsnorm_f32", "pointwise", "matmul", "attention"])
def test_large_runs_are_pipelined(irx, kir, shard, nshards, want):
    assert irx.compile(kir).host_chunks(shard, nshards) == want


@pytest.mark.parametrize("kir", [
    ka.reduce_all(1 << 26),                               # one output for the whole run
    ka.reduce_rows(65536, 4096),                          # 256 KB of output: nothing to overlap
    ka.softmax(64, 4096),                                 # too small to split
    ka.attention(1, 1, 1024, 128),                        # a single unit
], ids=["reduce_all", "reduce_rows", "small_softmax", "one_head"])
def test_other_runs_are_not(irx, kir):
    assert irx.compile(kir).host_chunks() == 1


def test_chunks_refuse_a_bad_shard(irx):
    plan = irx.compile(ka.softmax(8192, 4096))
    with pytest.raises(irx.IrxError):
        plan.host_chunks(2, 2)
