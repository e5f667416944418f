"""GPU parity of the load-time checkpoint kernel (torch.ops.grinqh.unpack_checkpoint,
C ABI grinqh_unpack_checkpoint): the compressed-tensors pack-quantized weight of a
shard -> this rank's int8 staging codes, bit-exact against the CPU oracle's codec
(itself pinned to compressed-tensors' pack_to_int32 by tests/golden), for every bit
width, ragged sizes, tensor-parallel slices and unaligned column offsets; and the
plugin's weight loader on CUDA (which runs this kernel) against its CPU path."""
import time

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import grinqh.kernel  # noqa: F401


def checkpoint_tensor(codes_nk, b):
    """The shard as stored in the checkpoint: int32 packed (int8 codes for b = 6)."""
    if b == 6:
        return torch.from_numpy(np.ascontiguousarray(codes_nk))
    return torch.from_numpy(O.ct_pack_to_int32(codes_nk, b))


@pytest.mark.parametrize("b", (2, 4, 8))
def test_golden_checkpoint_vectors(golden, b):
    """compressed-tensors' own pack_to_int32 output -> staging codes, bit-exact (b = 6
    checkpoints hold int8 codes, not packed words, so they have no packed vector)."""
    from grinqh.utils import unpack_checkpoint
    codes = golden[f"ct_codes_b{b}"]  # (N, K) as compressed-tensors' pack_to_int32 saw them
    src = torch.from_numpy(golden[f"ct_packed_b{b}"]).cuda()
    n, k = codes.shape
    dst = torch.full((k, n), 77, dtype=torch.int8, device="cuda")
    unpack_checkpoint(src, b, 0, n, 0, dst, 0)
    np.testing.assert_array_equal(dst.cpu().numpy(), codes.T)


@pytest.mark.parametrize("b", (2, 4, 6, 8))
@pytest.mark.parametrize("case", [
    # (rows_total, K_total, row0, rows, k0, k_local, n_cols of dst, n_off)
    (64, 128, 0, 64, 0, 128, 64, 0),
    (200, 384, 0, 200, 0, 384, 200, 0),        # ragged rows (not a multiple of the 64 tile)
    (512, 1024, 256, 128, 512, 512, 384, 96),   # column-parallel rows + row-parallel K slice
    (96, 256, 32, 48, 128, 128, 101, 53),       # odd destination width and offset (byte stores)
    (16, 4096, 0, 16, 0, 4096, 16, 0),          # long K, few rows
])
def test_slices_match_oracle(b, case):
    from grinqh.utils import unpack_checkpoint
    rows_total, k_total, row0, rows, k0, k_local, n_cols, n_off = case
    rng = np.random.default_rng(b * 1000 + rows_total)
    lo, hi = -(1 << (b - 1)), (1 << (b - 1))
    codes = rng.integers(lo, hi, size=(rows_total, k_total)).astype(np.int8)
    src = checkpoint_tensor(codes, b).cuda()
    dst = torch.full((k_local, n_cols), 99, dtype=torch.int8, device="cuda")
    unpack_checkpoint(src, b, row0, rows, k0, dst, n_off)
    got = dst.cpu().numpy()
    want = O.ct_unpack_from_int32(O.ct_pack_to_int32(codes, b), b, codes.shape) if b != 6 else codes
    np.testing.assert_array_equal(got[:, n_off:n_off + rows], want[row0:row0 + rows, k0:k0 + k_local].T)
    # nothing outside the written columns changed
    assert (got[:, :n_off] == 99).all() and (got[:, n_off + rows:] == 99).all()


def test_invalid_slices_raise():
    from grinqh.utils import unpack_checkpoint
    src = torch.zeros(64, 32, dtype=torch.int32, device="cuda")  # b = 8: 128 columns
    dst = torch.zeros(128, 64, dtype=torch.int8, device="cuda")
    with pytest.raises(RuntimeError):
        unpack_checkpoint(src, 8, 32, 64, 0, dst, 0)  # rows past the source
    with pytest.raises(RuntimeError):
        unpack_checkpoint(src, 8, 0, 64, 2, dst[:64], 0)  # k0 not a multiple of 4 fields
    with pytest.raises(RuntimeError):
        unpack_checkpoint(src, 8, 0, 64, 64, dst, 0)  # columns past the source row
    with pytest.raises(RuntimeError):
        unpack_checkpoint(src.float(), 8, 0, 64, 0, dst, 0)  # wrong source dtype


@pytest.mark.parametrize("b", (4, 6, 8))
def test_loader_on_cuda_matches_cpu_loader(b):
    """create_weights + weight_loader of a merged column-parallel layer (rank 1 of 2)
    on CUDA (the checkpoint kernel) and on CPU (the torch path) stage the same codes,
    and they are this rank's rows of each shard."""
    import vllm.model_executor.parameter as P
    from grinqh import grinqh as G

    rank, world = 1, 2
    old = (P.get_tensor_model_parallel_rank, P.get_tensor_model_parallel_world_size)
    P.get_tensor_model_parallel_rank = lambda: rank
    P.get_tensor_model_parallel_world_size = lambda: world
    try:
        rng = np.random.default_rng(b)
        K, parts_full = 512, [256, 128]  # gate / up shards of the full layer
        parts = [p // world for p in parts_full]
        ckpt = {i: rng.integers(-(1 << (b - 1)), 1 << (b - 1), size=(p, K)).astype(np.int8)
                for i, p in enumerate(parts_full)}
        staged = {}
        for dev in ("cpu", "cuda"):
            with torch.device(dev):
                layer = torch.nn.Module()
                layer.tp_rank, layer.tp_size = rank, world
                m = G.GRINQHLinearMethod(G.GRINQHConfig(thresholds={}, max_bits=b), [0.1, 0.2, 0.3, 0.4])
                m.create_weights(layer, K, parts, K, sum(parts_full), torch.bfloat16)
            wp = getattr(layer, layer.grinqh_weight_param_name)
            for i in range(2):
                wp.weight_loader(wp, checkpoint_tensor(ckpt[i], b), i)
            staged[dev] = wp.data.view(torch.int8).cpu().numpy().copy()
        np.testing.assert_array_equal(staged["cuda"], staged["cpu"])
        want = np.concatenate([ckpt[i][rank * parts[i]:(rank + 1) * parts[i]] for i in range(2)], axis=0).T
        np.testing.assert_array_equal(staged["cuda"], want)
    finally:
        P.get_tensor_model_parallel_rank, P.get_tensor_model_parallel_world_size = old


def test_checkpoint_kernel_is_faster_than_the_torch_path():
    """Load-time cost of one gate/up-sized shard (14336 x 4096, b = 8) already on the
    device: the kernel against compressed-tensors' unpack + narrow + transposed copy."""
    from compressed_tensors import unpack_from_int32
    from grinqh.utils import unpack_checkpoint
    n, k, b = 14336, 4096, 8
    src = torch.randint(-2**31, 2**31 - 1, (n, k * b // 32), dtype=torch.int32, device="cuda")
    dst = torch.empty(k, n, dtype=torch.int8, device="cuda")

    def kernel():
        unpack_checkpoint(src, b, 0, n, 0, dst, 0)

    def torch_path():
        w = unpack_from_int32(src, b, torch.Size((n, k)))
        dst.copy_(w.T.to(torch.int8))

    times = {}
    for name, fn in (("kernel", kernel), ("torch", torch_path)):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        times[name] = (time.perf_counter() - t0) / 5
    ref = dst.clone()
    kernel()
    torch.cuda.synchronize()
    assert torch.equal(dst, ref)
    moved = src.numel() * 4 + dst.numel()
    print(f"checkpoint shard {n}x{k} b={b}: kernel {times['kernel'] * 1e6:.0f} us "
          f"({moved / times['kernel'] / 1e9:.0f} GB/s), torch path {times['torch'] * 1e6:.0f} us")
    assert times["kernel"] < times["torch"]
