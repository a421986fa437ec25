"""CPU: host-side logic of the package against the reference's own outputs,
plus the C-ABI library's exports and host-side argument checks."""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as orc
from taomate_hd_b200 import build as native_build
from taomate_hd_b200 import capi as capi_mod
from taomate_hd_b200 import dit
from taomate_hd_b200.parallel import ParallelContext, current_parallel_context, use_parallel_context

GOLDEN = Path(__file__).resolve().parent / "golden"


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


@pytest.fixture(scope="module")
def ref():
    return np.load(GOLDEN / "reference_host.npz"), json.loads((GOLDEN / "reference_host.json").read_text())


# ------------------------------------------------------------------ sharding
@pytest.mark.parametrize("tp", [1, 2, 4])
def test_tp_sharding_matches_reference(ref, tp):
    """dit.column_slice / row_slice give the reference's shards: merged QKV
    per projection, a plain column weight, the row K slice, and the LoRA B /
    A shards (distributed/linear.py:161-225, :291-296; lora_checkpoint.py:73-97)."""
    arrays, _ = ref
    full_qkv, full_row = _bf16(arrays["shard.full_qkv"]), _bf16(arrays["shard.full_row"])
    full_bias = _bf16(arrays["shard.full_bias"])
    lora_b, lora_a = torch.from_numpy(arrays["shard.lora_b"]), torch.from_numpy(arrays["shard.lora_a"])
    sizes = (48, 48, 48)
    for rank in range(tp):
        key = f"shard.tp{tp}.r{rank}"
        assert torch.equal(dit.column_slice(full_qkv, tp, rank, sizes), _bf16(arrays[f"{key}.merged_w"]))
        assert torch.equal(dit.column_slice(full_bias, tp, rank, sizes), _bf16(arrays[f"{key}.merged_b"]))
        assert torch.equal(dit.column_slice(full_qkv, tp, rank), _bf16(arrays[f"{key}.column_w"]))
        assert torch.equal(dit.row_slice(full_row, tp, rank), _bf16(arrays[f"{key}.row_w"]))
        assert torch.equal(dit.column_slice(lora_b, tp, rank, sizes), torch.from_numpy(arrays[f"{key}.lora_b"]))
        assert torch.equal(dit.row_slice(lora_a, tp, rank), torch.from_numpy(arrays[f"{key}.lora_a"]))
        # the oracle's restatement agrees with the package's helpers
        assert torch.equal(orc.merged_column_shard(full_qkv, sizes, tp, rank),
                           dit.column_slice(full_qkv, tp, rank, sizes))
        assert torch.equal(orc.row_shard(full_row, tp, rank), dit.row_slice(full_row, tp, rank))


def test_shape_errors():
    with pytest.raises(ValueError, match="divide"):
        dit.column_slice(torch.zeros(10, 8), 4, 0)
    with pytest.raises(ValueError, match="divide"):
        dit.column_slice(torch.zeros(14, 8), 4, 0, (8, 6))
    with pytest.raises(ValueError, match="add up"):
        dit.column_slice(torch.zeros(16, 8), 2, 0, (8, 6))
    with pytest.raises(ValueError, match="divide"):
        dit.row_slice(torch.zeros(8, 9), 2, 1)


def test_parallel_context_validation():
    with pytest.raises(ValueError):
        ParallelContext(tp_world_size=2, tp_rank=0)          # group required
    with pytest.raises(ValueError):
        ParallelContext(tp_world_size=2, tp_rank=2, tp_group=object())
    ctx = ParallelContext(tp_world_size=2, tp_rank=1, tp_group=object())
    assert current_parallel_context().tp_world_size == 1
    with use_parallel_context(ctx):
        assert current_parallel_context() is ctx
    assert current_parallel_context().tp_world_size == 1
    with pytest.raises(TypeError):
        with use_parallel_context("nope"):
            pass


# ------------------------------------------------------------------ LoRA
@pytest.mark.parametrize("which", ["qkv", "out"])
def test_oracle_lora_matches_reference_wrapper(ref, which):
    """The oracle's LoRA composition equals the reference wrapper's forward
    (H3InferenceParallelLinearLoRA at TP=1 on a BF16 base,
    lora_checkpoint.py:126-154), bit for bit."""
    arrays, meta = ref
    x = _bf16(arrays["lora.x"])
    base = torch.nn.functional.linear(x, _bf16(arrays[f"lora.{which}_w"]))
    y = orc.lora_column(base, x, _bf16(arrays[f"lora.{which}_a"]), _bf16(arrays[f"lora.{which}_b"]),
                        float(arrays["lora.scale"]))
    assert torch.equal(y, _bf16(arrays[f"lora.{which}_y"]))
    assert meta["lora_receipt"]["scale"] == float(arrays["lora.scale"])


# ------------------------------------------------------------------ streamed weight conversion
def test_quantize_weight_into_validates_before_any_launch():
    """The streamed W8 conversion checks dtypes, shapes and the staging bound
    on the host (the reference's load_cutlass_w8a8_stream_weight_ raises
    TypeError / ValueError for the same cases, w8a8.py:207-242)."""
    from taomate_hd_b200 import ops

    src = torch.zeros(4, 16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize_weight_int8_into(torch.empty(4, 16, dtype=torch.int8), torch.empty(4, 1), src)

    class FakeCuda:
        """Stands in for a device tensor so the host checks run on CPU."""

        def __init__(self, t):
            self.t, self.is_cuda = t, True
            self.dtype, self.shape = t.dtype, t.shape

        def numel(self):
            return self.t.numel()

        def is_contiguous(self):
            return self.t.is_contiguous()

    q, s = FakeCuda(torch.empty(4, 16, dtype=torch.int8)), FakeCuda(torch.empty(4, 1))
    with pytest.raises(TypeError):
        ops.quantize_weight_int8_into(q, s, torch.zeros(4, 16, dtype=torch.int32))
    with pytest.raises(ValueError, match="same 2-D shape"):
        ops.quantize_weight_int8_into(q, s, torch.zeros(4, 8, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="one element per output row"):
        ops.quantize_weight_int8_into(q, FakeCuda(torch.empty(3)), src)
    with pytest.raises(ValueError, match="staging_bytes"):
        ops.quantize_weight_int8_into(q, s, src, staging_bytes=0)


# ------------------------------------------------------------------ native library
def test_build_is_current():
    assert native_build.is_current(), "run `python -m taomate_hd_b200.build`"


def test_torch_op_library_links_shared_libstdcxx():
    """The op library must use the process's libstdc++: a statically linked
    copy has its own locale state and crashes while formatting the first
    error message an op raises."""
    import shutil
    import subprocess

    from taomate_hd_b200 import build

    if shutil.which("readelf") is None:
        pytest.skip("readelf not available")
    dyn = subprocess.run(["readelf", "-d", str(build.TORCH_SO)], capture_output=True, text=True)
    assert dyn.returncode == 0
    assert "libstdc++.so" in dyn.stdout
    syms = subprocess.run(["readelf", "--dyn-syms", "--wide", str(build.TORCH_SO)],
                          capture_output=True, text=True).stdout
    assert "_ZNSo9_M_insertIlEERSoT_" not in [line.split()[-1] for line in syms.splitlines()
                                               if " DEFAULT " in line and " UND " not in line]


def test_c_abi_exports_every_header_symbol():
    lib = ctypes.CDLL(str(native_build.CAPI_SO))
    names = capi_mod.header_symbols()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(capi_mod.SIGNATURES), "ctypes signatures out of sync with the header"


def test_c_abi_host_argument_checks():
    from taomate_hd_b200 import _native

    lib = _native.capi()
    assert lib.tm_version() >= 100
    assert capi_mod.status_string(lib, 0) == "ok"
    p = ctypes.c_void_p(1 << 20)  # never dereferenced: every call below fails validation first
    quant = lib.tm_dynamic_scaled_int8_quant
    assert quant(p, p, 0, p, None, 4, 64, 32, None) == capi_mod.TM_ERR_SHAPE       # ld < cols
    assert quant(p, p, 0, p, None, -1, 64, 64, None) == capi_mod.TM_ERR_SHAPE
    assert quant(p, p, 7, p, None, 4, 64, 64, None) == capi_mod.TM_ERR_DTYPE
    assert quant(None, p, 0, p, None, 4, 64, 64, None) == capi_mod.TM_ERR_NULL_POINTER
    assert quant(p, p, 0, p, p, 4, 64, 64, None) == capi_mod.TM_ERR_UNSUPPORTED     # azp
    assert quant(p, p, 0, p, None, 0, 64, 64, None) == capi_mod.TM_OK               # no rows
    mm = lib.tm_cutlass_scaled_mm
    args = dict(m=128, n=256, k=512)
    assert mm(p, 0, p, p, p, 128, p, 256, None, 128, 256, 500, 512, 512, 256, None) == capi_mod.TM_ERR_SHAPE
    assert mm(p, 0, p, p, p, 128, p, 256, None, 128, 250, 512, 512, 512, 256, None) == capi_mod.TM_ERR_SHAPE
    assert mm(p, 5, p, p, p, 128, p, 256, None, 128, 256, 512, 512, 512, 256, None) == capi_mod.TM_ERR_DTYPE
    assert mm(p, 0, p, p, p, 7, p, 256, None, 128, 256, 512, 512, 512, 256, None) == capi_mod.TM_ERR_SHAPE
    assert mm(p, 0, p, p, p, 128, p, 256, None, 128, 256, 512, 520, 512, 256, None) == capi_mod.TM_ERR_ALIGNMENT
    assert mm(p, 0, p, p, p, 1, p, 256, None, 0, 256, 512, 512, 512, 256, None) == capi_mod.TM_OK
    assert mm(p, 0, None, p, p, 128, p, 256, None, 128, 256, 512, 512, 512, 256, None) == capi_mod.TM_ERR_NULL_POINTER
    assert args  # sizes used above
    tile = lib.tm_scaled_mm_i8_tile
    assert tile(p, 0, p, p, p, 128, p, 256, None, 128, 256, 512, 512, 512, 256, 0, None, 96, None) == capi_mod.TM_ERR_UNSUPPORTED
    arr = (ctypes.c_void_p * 2)(p, p)
    # fused row-parallel LoRA: LoRA operand checks, then the scatter checks
    lrs = lib.tm_scaled_mm_i8_lora_reduce_scatter
    lar = lib.tm_scaled_mm_i8_lora_all_reduce
    #         out a  b  sa  n    sb  n    bias t  ldt lb ldlb r   m    n    k    lda  ldb  ldo  part flags w  rank ep st
    assert lrs(p, p, p, p, 512, p, 768, None, p, 64, p, 64, 12, 512, 768, 256, 256, 256, 768, arr, arr,
               2, 0, 1, None) == capi_mod.TM_ERR_UNSUPPORTED  # rank not a multiple of 8
    assert lrs(p, p, p, p, 500, p, 768, None, p, 64, p, 64, 64, 500, 768, 256, 256, 256, 768, arr, arr,
               2, 0, 1, None) == capi_mod.TM_ERR_SHAPE  # rows not a multiple of 256 x world
    assert lrs(p, p, p, p, 512, p, 768, None, p, 64, p, 64, 64, 512, 768, 256, 256, 256, 768, arr, arr,
               9, 0, 1, None) == capi_mod.TM_ERR_TOO_LARGE
    assert lar(p, p, p, 512, p, 768, None, p, 64, p, 64, 64, 512, 768, 256, 256, 256, arr, arr, None,
               2, 0, 1, None) == capi_mod.TM_ERR_NULL_POINTER  # no output buffers
    assert lar(p, p, p, 512, p, 768, None, p, 60, p, 64, 64, 512, 768, 256, 256, 256, arr, arr, arr,
               2, 0, 1, None) == capi_mod.TM_ERR_SHAPE  # ldt below the rank
    # Ulysses exchange over NVLink
    ux = lib.tm_scaled_mm_i8_ulysses_exchange
    #        a  b  sa  n    sb  n     bias  m    n     k    lda  ldb  heads hd  recv flags w  rank ep st
    assert ux(p, p, p, 256, p, 3072, None, 256, 3072, 512, 512, 512, 8, 128, None, arr, 2, 0, 1,
              None) == capi_mod.TM_ERR_NULL_POINTER
    assert ux(p, p, p, 256, p, 3072, None, 256, 3072, 512, 512, 512, 8, 128, arr, arr, 2, 2, 1,
              None) == capi_mod.TM_ERR_SHAPE  # rank outside the group
    assert ux(p, p, p, 256, p, 1536, None, 256, 1536, 512, 512, 512, 16, 32, arr, arr, 2, 0, 1,
              None) == capi_mod.TM_ERR_SHAPE  # head_dim not a multiple of 64
    assert ux(p, p, p, 250, p, 3072, None, 250, 3072, 512, 512, 512, 8, 128, arr, arr, 2, 0, 1,
              None) == capi_mod.TM_ERR_SHAPE  # tokens not a multiple of 32
    down = lib.tm_lora_down_proj  # (t, ldt, x, ldx, a, lda, rank, m, k, stream)
    assert down(p, 64, p, 512, p, 512, 64, 0, 512, None) == capi_mod.TM_OK            # no rows
    assert down(p, 72, p, 512, p, 512, 72, 128, 512, None) == capi_mod.TM_ERR_UNSUPPORTED
    assert down(p, 64, p, 512, p, 512, 12, 128, 512, None) == capi_mod.TM_ERR_UNSUPPORTED
    assert down(p, 32, p, 512, p, 512, 64, 128, 512, None) == capi_mod.TM_ERR_SHAPE  # ldt < rank
    assert down(p, 64, p, 500, p, 512, 64, 128, 512, None) == capi_mod.TM_ERR_SHAPE  # ldx < k
    assert down(p, 64, p, 516, p, 512, 64, 128, 512, None) == capi_mod.TM_ERR_ALIGNMENT
    assert down(ctypes.c_void_p((1 << 20) + 8), 64, p, 512, p, 512, 64, 128, 512,
                None) == capi_mod.TM_ERR_ALIGNMENT
    assert down(None, 64, p, 512, p, 512, 64, 128, 512, None) == capi_mod.TM_ERR_NULL_POINTER


def test_torch_ops_have_no_cpu_path():
    from taomate_hd_b200 import ops

    assert hasattr(torch.ops.taomate_w8a8, "cutlass_scaled_mm")
    with pytest.raises(RuntimeError):
        ops.scaled_int8_quant(torch.randn(4, 16, dtype=torch.bfloat16))
    with pytest.raises(NotImplementedError):
        torch.ops.taomate_w8a8.dynamic_scaled_int8_quant(
            torch.empty(4, 16, dtype=torch.int8), torch.randn(4, 16, dtype=torch.bfloat16),
            torch.empty(4, 1), None)


def test_stale_build_is_refused(monkeypatch):
    from taomate_hd_b200 import _native

    monkeypatch.setattr(native_build, "source_digest", lambda: "not-the-stamp")
    with pytest.raises(_native.NativeLibraryError):
        _native._require_current()


def test_ops_module_passes_the_reference_backend_check():
    """The reference's loader imports the backend by module name and requires
    callable scaled_int8_quant and cutlass_scaled_mm (w8a8.py:76-86); its
    workspace requires the two out-variant ops in the op namespace
    (w8a8.py:22-29)."""
    import importlib

    backend = importlib.import_module("taomate_hd_b200.ops")
    for name in ("scaled_int8_quant", "cutlass_scaled_mm"):
        assert callable(getattr(backend, name, None)), name
    namespace = getattr(torch.ops, "taomate_w8a8")
    for name in ("dynamic_scaled_int8_quant", "cutlass_scaled_mm"):
        assert callable(getattr(namespace, name, None)), name


def _tile_coords(tile, num_m, num_n, m_owners, mb_per_owner, group_m=16, group_n=0):
    """Restatement of the GEMM's tile_coords (grouped raster: M-block groups,
    or N-block groups for long K; then the owner-interleaved M order of the
    fused reduce-scatter / all-reduce)."""
    if group_n > 0:
        group_size = group_n * num_m
        group = tile // group_size
        first_n = group * group_n
        gn = min(num_n - first_n, group_n)
        local = tile - group * group_size
        mb, nb = local // gn, first_n + local % gn
    else:
        group_size = group_m * num_n
        group = tile // group_size
        first_m = group * group_m
        gm = min(num_m - first_m, group_m)
        local = tile - group * group_size
        mb, nb = first_m + local % gm, local // gm
    if m_owners > 1:
        mb = (mb % m_owners) * mb_per_owner + mb // m_owners
    return mb, nb


@pytest.mark.parametrize("m,n,world,rows_per_mb,bn,ctas", [
    (8192, 3072, 8, 256, 256, 74),    # fc2 at TP=8, CTA-pair tiles
    (8192, 3072, 2, 256, 256, 74),
    (20480, 3072, 8, 256, 256, 74),   # 768p out-proj at TP=8
    (20480, 3072, 4, 128, 128, 148),  # one-CTA tiles
    (2048, 1000, 2, 128, 64, 148),    # ragged N, one partial raster group
])
def test_interleaved_tile_order_is_a_permutation_covering_all_owners(m, n, world, rows_per_mb,
                                                                     bn, ctas):
    num_m, num_n = m // rows_per_mb, -(-n // bn)
    mb_per_owner = (m // world) // rows_per_mb
    assert num_m == world * mb_per_owner  # the host's m % (world x 256) check guarantees it
    tiles = [_tile_coords(t, num_m, num_n, world, mb_per_owner) for t in range(num_m * num_n)]
    assert sorted(tiles) == [(a, b) for a in range(num_m) for b in range(num_n)]
    owner_of = [mb // mb_per_owner for mb, _ in tiles]
    # every full wave of concurrent tiles sends to every owner, nearly evenly
    for w0 in range(0, len(tiles) - ctas + 1, ctas):
        counts = np.bincount(owner_of[w0:w0 + ctas], minlength=world)
        assert counts.min() > 0 and counts.max() - counts.min() <= max(2, ctas // world // 2)
    # without the interleave a wave covers only a few owners (what it fixes)
    plain = [_tile_coords(t, num_m, num_n, 0, 0)[0] // mb_per_owner for t in range(ctas)]
    assert len(set(plain)) <= -(-16 // mb_per_owner) + 1 < world or world <= 2


@pytest.mark.parametrize("world,rows,cols,match", [
    (9, 8192, 3072, "1..8 ranks"),
    (2, 8192 + 256, 3072, "multiple of 256"),
    (8, 1024, 3072, "multiple of 256"),
    (2, 8192, 3080, "multiple of 16"),
])
def test_peer_reduce_rejects_unsupported_shapes_before_allocating(world, rows, cols, match):
    """Shape checks of the fused row-parallel reduction run on the host before
    any allocation or collective, identically on every rank."""
    from types import SimpleNamespace

    from taomate_hd_b200.peer_reduce import PeerAllReduce, PeerReduceScatter

    ctx = SimpleNamespace(tp_world_size=world, tp_rank=0, tp_group=None)
    for cls in (PeerReduceScatter, PeerAllReduce):
        with pytest.raises(ValueError, match=match):
            cls(ctx, rows, cols, torch.device("cpu"))


def test_ulysses_errors_match_reference_before_any_launch():
    """merged_qkv_sequence_to_heads (distributed/ulysses.py:166-197): a weight
    that is not 3 x heads x head_dim rows raises ValueError, and an exchange
    without torch.distributed raises RuntimeError."""
    from taomate_hd_b200.ulysses import exchange_qkv, merged_qkv_sequence_to_heads_w8a8

    q = torch.zeros(64, 256, dtype=torch.int8)
    s = torch.ones(64, 1)
    w = torch.zeros(3 * 4 * 128, 256, dtype=torch.int8)
    ws = torch.ones(3 * 4 * 128)
    with pytest.raises(ValueError, match="merged QKV width"):
        merged_qkv_sequence_to_heads_w8a8(q, s, w, ws, None, num_heads=4, head_dim=64)
    assert not torch.distributed.is_initialized()
    with pytest.raises(RuntimeError, match="initialized torch.distributed"):
        merged_qkv_sequence_to_heads_w8a8(q, s, w, ws, None, num_heads=4, head_dim=128, world=2)
    with pytest.raises(RuntimeError, match="initialized torch.distributed"):
        exchange_qkv(torch.zeros(2, 3, 4, 2, 8, dtype=torch.bfloat16))


def _choose_group_n(num_n, rows_per_mb, bn, k, group_m=16):
    """Restatement of the host's choose_group_n (24 MiB of A panels, 48 MiB of B)."""
    if group_m * rows_per_mb * k <= 24 << 20:
        return 0
    return max(1, min(num_n, (48 << 20) // (bn * k)))


@pytest.mark.parametrize("m,n,k,rows_per_mb,bn,world", [
    (8192, 3072, 12288, 256, 256, 0),    # 480p fc2 at TP=1: N-fastest groups
    (8192, 3072, 12288, 256, 256, 2),    # owner interleave on top
    (8192, 3072, 6144, 256, 256, 2),     # fc2 at TP=2: 24 MiB of A panels, M-groups
    (20480, 12288, 12288, 256, 256, 0),  # B does not fit: groups of a few N-blocks
    (8192, 12288, 3072, 256, 256, 0),    # fc1: short K keeps M-groups
    (1000, 3000, 16384, 128, 64, 0),     # ragged M and N
])
def test_long_k_raster_is_a_permutation(m, n, k, rows_per_mb, bn, world):
    num_m, num_n = -(-m // rows_per_mb), -(-n // bn)
    group_n = _choose_group_n(num_n, rows_per_mb, bn, k)
    assert (group_n == 0) == (k <= 6144)
    mb_per_owner = num_m // world if world else 0
    tiles = [_tile_coords(t, num_m, num_n, world, mb_per_owner, group_n=group_n)
             for t in range(num_m * num_n)]
    assert sorted(tiles) == [(a, b) for a in range(num_m) for b in range(num_n)]
    if group_n:
        # a wave of 74 pair tiles touches few A panels and stays in one N-group
        wave = tiles[:74]
        assert len({mb for mb, _ in wave}) <= -(-74 // min(group_n, num_n)) + 1


def _ul_peer_address(col: int, row: int, src: int, m: int, heads: int, head_dim: int,
                     world: int) -> tuple[int, int]:
    """Restatement of the exchange epilogue's store address (ul_peer_dest,
    ul_peer_base and the row offset in gemm_i8.cu): output column `col` of
    token `row` on source rank `src` lands in destination `w`'s receive buffer
    [world, 3, m, local x head_dim] at flat element `offset`."""
    local = -(-heads // world)
    width = heads * head_dim
    qkv, within = divmod(col, width)
    head = within // head_dim
    w = head // local
    x = within - w * local * head_dim
    ld = local * head_dim
    return w, ((src * 3 + qkv) * m + row) * ld + x


@pytest.mark.parametrize("heads,head_dim,world,m", [(8, 128, 2, 64), (9, 128, 2, 32),
                                                     (24, 128, 8, 32), (6, 64, 4, 32),
                                                     (2, 128, 4, 32)])
def test_ulysses_exchange_addresses_equal_send_layout_then_all_to_all(heads, head_dim, world, m):
    """Every source's outputs land exactly where the reference's send layout
    followed by all_to_all_single puts them (rank w receives chunk w of every
    source, in source order), each real position once, padded heads never."""
    from oracle import w8a8_oracle as orc

    n = 3 * heads * head_dim
    local = -(-heads // world)
    # value[src][row, col] = a unique tag per (src, row, col)
    tags = [torch.arange(m * n, dtype=torch.float64).reshape(m, n) + src * m * n
            for src in range(world)]
    # reference: send layout per source, then all-to-all (chunk w of src -> rank w, slot src)
    sends = [orc.merged_qkv_send_layout(t, heads, head_dim, world) for t in tags]
    want = [torch.stack([sends[src][w] for src in range(world)]) for w in range(world)]
    got = [torch.full((world, 3, m, local, head_dim), -1.0, dtype=torch.float64)
           for _ in range(world)]
    flat = [g.view(-1) for g in got]
    written = [torch.zeros(g.numel(), dtype=torch.int64) for g in got]
    cols = torch.arange(n)
    for src in range(world):
        for row in range(m):
            for c0 in range(0, n, 64):  # one address computation per 64-column pass
                w, off = _ul_peer_address(c0, row, src, m, heads, head_dim, world)
                flat[w][off:off + 64] = tags[src][row, c0:c0 + 64]
                written[w][off:off + 64] += 1
    assert cols.numel() == n
    for w in range(world):
        real = max(0, min(local, heads - w * local))
        mask = torch.zeros(world, 3, m, local, head_dim, dtype=torch.bool)
        mask[:, :, :, :real, :] = True
        assert bool((written[w].view_as(mask)[mask] == 1).all())   # each real position once
        assert bool((written[w].view_as(mask)[~mask] == 0).all())  # padded heads untouched
        assert torch.equal(got[w][mask], want[w][mask])
        assert bool((want[w][~mask] == 0).all())  # the reference pads with zero heads


@pytest.mark.parametrize("tokens,head_dim,match", [(250, 128, "multiple of 32"),
                                                   (256, 96, "multiple of 64")])
def test_ulysses_exchange_rejects_unsupported_shapes_before_allocating(tokens, head_dim, match):
    """The NVLink exchange's shape rules raise before any buffer is allocated,
    through the explicit-group constructor and through a ParallelContext's
    Ulysses axis."""
    from taomate_hd_b200.parallel import ParallelContext
    from taomate_hd_b200.ulysses import PeerUlyssesExchange

    with pytest.raises(ValueError, match=match):
        PeerUlyssesExchange(tokens, 8, head_dim, torch.device("cpu"), group=object(), world=2,
                            rank=1)
    ctx = ParallelContext(ulysses_world_size=2, ulysses_rank=0, ulysses_group=object())
    with pytest.raises(ValueError, match=match):
        PeerUlyssesExchange.from_context(ctx, tokens, 8, head_dim, torch.device("cpu"))


def test_peer_lora_operands_are_checked_before_any_launch():
    """The fused row-parallel LoRA calls refuse LoRA operands whose extents
    differ from the ones the kernel's tensor maps assume (a shorter lora_t
    would be read past its end), before anything reaches the device."""
    from taomate_hd_b200.peer_reduce import _check_lora

    with pytest.raises(RuntimeError, match="CUDA"):  # host tensors
        _check_lora(torch.empty(512, 64, dtype=torch.bfloat16),
                    torch.empty(768, 64, dtype=torch.bfloat16), 512, 768)

    class _Cuda:  # tensor metadata of a CUDA tensor; never dereferenced
        def __init__(self, shape, dtype=torch.bfloat16, stride1=1):
            self.shape, self.dtype = torch.Size(shape), dtype
            self.device = torch.device("cuda", 0)
            self._stride1 = stride1

        def dim(self):
            return len(self.shape)

        def stride(self, i):
            return self._stride1

    assert _check_lora(_Cuda((512, 64)), _Cuda((768, 64)), 512, 768) == 64
    with pytest.raises(ValueError, match=r"lora_t must be \[512, r\]"):
        _check_lora(_Cuda((256, 64)), _Cuda((768, 64)), 512, 768)
    with pytest.raises(ValueError, match="lora_t must be"):
        _check_lora(_Cuda((512, 64)), _Cuda((768, 32)), 512, 768)
    with pytest.raises(ValueError, match="multiple of 8"):
        _check_lora(_Cuda((512, 12)), _Cuda((768, 12)), 512, 768)
    with pytest.raises(ValueError, match="bfloat16"):
        _check_lora(_Cuda((512, 64), torch.float16), _Cuda((768, 64)), 512, 768)
    with pytest.raises(ValueError, match="contiguous"):
        _check_lora(_Cuda((512, 64), stride1=2), _Cuda((768, 64)), 512, 768)


def test_peer_gemm_operands_are_checked_before_any_launch():
    """The fused calls (reduce-scatter, all-reduce, their LoRA forms, the
    Ulysses exchange) refuse operands whose dtype, layout or length differ
    from what the kernels read, before anything reaches the device."""
    from taomate_hd_b200.peer_reduce import _check_operands

    class _T:  # tensor metadata of a CUDA tensor; never dereferenced
        def __init__(self, shape, dtype, contiguous=True, stride1=1, device="cuda"):
            self.shape, self.dtype = torch.Size(shape), dtype
            self.device = torch.device(device, 0) if device == "cuda" else torch.device(device)
            self._c, self._s1 = contiguous, stride1

        def dim(self):
            return len(self.shape)

        def stride(self, i):
            return self._s1

        def is_contiguous(self):
            return self._c

        def numel(self):
            n = 1
            for d in self.shape:
                n *= d
            return n

    i8, f32, bf = torch.int8, torch.float32, torch.bfloat16
    ok = dict(q=_T((512, 256), i8), q_scale=_T((512, 1), f32), w_q=_T((768, 256), i8),
              w_scale=_T((768,), f32), bias=_T((768,), bf))
    assert _check_operands(**ok, rows=512, cols=768) == (512, 256)
    assert _check_operands(**{**ok, "bias": None, "q_scale": _T((1,), f32)},
                           rows=512, cols=768) == (512, 256)
    bad = [({"q": _T((512, 256), bf)}, ValueError, "int8"),
           ({"q": _T((512, 256), i8, device="cpu")}, RuntimeError, "CUDA"),
           ({"w_q": _T((768, 256), i8, stride1=2)}, ValueError, "contiguous"),
           ({"w_q": _T((768, 128), i8)}, ValueError, "shape differs"),
           ({"q": _T((256, 256), i8)}, ValueError, "shape differs"),
           ({"q_scale": _T((256, 1), f32)}, ValueError, "q_scale"),
           ({"w_scale": _T((768,), bf)}, ValueError, "w_scale"),
           ({"w_scale": _T((768,), f32, contiguous=False)}, ValueError, "w_scale"),
           ({"bias": _T((512,), bf)}, ValueError, "bias"),
           ({"bias": _T((768,), torch.float16)}, ValueError, "bias"),
           ({"bias": _T((768,), bf, device="cpu")}, RuntimeError, "CUDA")]
    for change, exc, match in bad:
        with pytest.raises(exc, match=match):
            _check_operands(**{**ok, **change}, rows=512, cols=768)


def test_peer_reduce_scatter_output_and_failed_call_latch():
    """The reduce-scatter output must be this rank's bf16 [rows/world, cols]
    block with contiguous rows on CUDA; after a native call fails on one rank
    its call count no longer matches the other ranks', so the buffers refuse
    further calls instead of pairing this rank's next call with the wrong
    call of its peers."""
    from types import SimpleNamespace

    from taomate_hd_b200.peer_reduce import PeerReduceScatter, _PeerBuffers

    class _Out:  # tensor metadata; never dereferenced
        def __init__(self, shape, dtype=torch.bfloat16, stride1=1, device="cuda"):
            self.shape, self.dtype, self._s1 = torch.Size(shape), dtype, stride1
            self.device = torch.device(device, 0) if device == "cuda" else torch.device(device)

        def stride(self, i):
            return self._s1

    me = SimpleNamespace(rows_per_owner=256, cols=768)
    PeerReduceScatter._check_out(me, _Out((256, 768)))
    for out, exc in ((_Out((512, 768)), ValueError), (_Out((256, 768), torch.float16), ValueError),
                     (_Out((256, 768), stride1=2), ValueError),
                     (_Out((256, 768), device="cpu"), RuntimeError)):
        with pytest.raises(exc):
            PeerReduceScatter._check_out(me, out)

    lib = SimpleNamespace(tm_status_string=lambda rc: b"CUDA error")
    bufs = SimpleNamespace(_failed=False, calls=0, _uses=[0, 0], _lib=lib)
    with pytest.raises(RuntimeError, match="CUDA error"):
        _PeerBuffers._raise(bufs, "tm_scaled_mm_i8_reduce_scatter", 5)
    assert bufs._failed and bufs.calls == 0
    with pytest.raises(RuntimeError, match="earlier call"):
        _PeerBuffers._next_set(bufs)
    assert bufs.calls == 0 and bufs._uses == [0, 0]


def test_documented_api_names_exist():
    """Every operator, class, torch op and C entry point that INTEGRATION.md
    and README.md tell a user to call exists under that name."""
    import re
    from pathlib import Path

    import taomate_hd_b200.dit as dit_mod
    import taomate_hd_b200.fused_kernels as fused_mod
    import taomate_hd_b200.ops as ops_mod
    import taomate_hd_b200.peer_reduce as peer_mod
    import taomate_hd_b200.ulysses as ulysses_mod

    root = Path(__file__).resolve().parents[1]
    text = (root / "INTEGRATION.md").read_text() + (root / "README.md").read_text()
    modules = {"ops": ops_mod, "ulysses": ulysses_mod, "peer_reduce": peer_mod, "dit": dit_mod,
               "fused_kernels": fused_mod}
    pattern = r"(?<![\w.])(ops|ulysses|peer_reduce|dit|fused_kernels)\.([A-Za-z_]\w*)"
    missing = [f"{m}.{name}" for m, name in re.findall(pattern, text)
               if name != "py" and not hasattr(modules[m], name)]
    for name in ("TPW8A8AttnProj", "TPW8A8LoRABlockStack"):  # listed after dit.TPW8A8MLP
        if name in text and not hasattr(dit_mod, name):
            missing.append(f"dit.{name}")
    for name in set(re.findall(r"torch\.ops\.taomate_w8a8\.(\w+)", text)):
        try:
            getattr(torch.ops.taomate_w8a8, name)
        except (AttributeError, RuntimeError):
            missing.append(f"torch.ops.taomate_w8a8.{name}")
    header = (root / "include" / "taomate_w8a8.h").read_text()
    missing += [name for name in set(re.findall(r"\btm_\w+", text)) if name not in header]
    assert not missing, missing
