"""CPU: the C ABI library loads, exports every entry point the header
declares, validates arguments like the reference, and plans launches -- all
without a GPU (no compute calls)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from decodekernels_b200 import capi

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "dk_paged_attention.h"


def _declared():
    text = HEADER.read_text()
    return re.findall(r"DK_API\s+[\w\s\*]+?\b(dk_\w+)\s*\(", text)


def test_header_declares_the_bound_entry_points():
    assert set(_declared()) == set(capi.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = capi.load()
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (dk_\w+)", out))
    assert set(_declared()) <= exported
    assert capi.version() == 800


def test_struct_layout_matches_header(tmp_path):
    """The ctypes mirrors have the C compiler's size and field offsets for
    include/dk_paged_attention.h."""
    # 10 pointers + 11 int64 + 12 int32 + 3 float = 228 bytes, padded to 232 (8-byte alignment)
    assert ctypes.sizeof(capi.DkPagedAttnArgs) == 232
    assert ctypes.sizeof(capi.DkPlan) == 40
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "dk_paged_attention.h"', "int main(void) {"]
    structs = (("DkPagedAttnArgs", capi.DkPagedAttnArgs), ("DkPlan", capi.DkPlan),
               ("DkCacheWriteArgs", capi.DkCacheWriteArgs), ("DkLseMergeArgs", capi.DkLseMergeArgs),
               ("DkPeerExchangeArgs", capi.DkPeerExchangeArgs), ("DkPeerGatherArgs", capi.DkPeerGatherArgs))
    for struct, cls in structs:
        lines.append(f'  printf("{struct} sizeof %zu\\n", sizeof({struct}));')
        for name, _ in cls._fields_:
            lines.append(f'  printf("{struct} {name} %zu\\n", offsetof({struct}, {name}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    include = Path(__file__).resolve().parents[1] / "include"
    subprocess.run(["gcc", "-std=c99", "-I", str(include), str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                               check=True).stdout.splitlines())
    for struct, cls in structs:
        assert int(got[f"{struct} sizeof"]) == ctypes.sizeof(cls)
        for name, _ in cls._fields_:
            assert int(got[f"{struct} {name}"]) == getattr(cls, name).offset, (struct, name)


def _args(**over):
    """CPU tensors only provide shapes/strides/pointers; nothing is launched."""
    n, hq, hkv, d, bs = over.pop("n", 4), over.pop("hq", 32), over.pop("hkv", 8), over.pop("d", 128), over.pop("bs", 16)
    dtype = over.pop("dtype", torch.bfloat16)
    q = torch.zeros(n, hq, d, dtype=dtype)
    k = torch.zeros(64, bs, hkv, d, dtype=dtype)
    bt = torch.zeros(max(n, 1), 64, dtype=torch.int32)
    sl = torch.zeros(max(n, 1), dtype=torch.int32)
    out = torch.zeros_like(q)
    max_seq_len = over.pop("max_seq_len", 513)
    ws = over.pop("ws", None)
    a = capi.make_args(q, k, k, bt, sl, d**-0.5, max_seq_len, out, ws, over.pop("partition_size", 0),
                       over.pop("force_simt", False))
    for key, val in over.items():
        setattr(a, key, val)
    return a


def _plan(a):
    p = capi.DkPlan()
    rc = capi.load().dk_plan(ctypes.byref(a), ctypes.byref(p))
    return rc, p.as_dict()


@pytest.mark.parametrize(
    "override,msg",
    [
        (dict(hq=128, hkv=8), "GQA group"),
        (dict(d=96), "head_dim"),
        (dict(hq=12, hkv=8), "multiple of num_kv_heads"),
        (dict(max_seq_len=-1), "max_seq_len"),
        (dict(dtype_code=7), "float16 or bfloat16"),
        (dict(k_stride_token=130), "multiples of head_dim / 32"),
        (dict(partition_size=100), "partition_size"),
        (dict(num_seqs=70000), "num_seqs"),
    ],
)
def test_validation_rejects_like_reference(override, msg):
    if "dtype_code" in override:
        a = _args()
        a.dtype = override["dtype_code"]
    else:
        a = _args(**override)
    rc, _ = _plan(a)
    assert rc == 1  # cudaErrorInvalidValue
    assert msg in capi.last_error()
    # the launch entry point rejects the same way, before touching the GPU
    assert capi.load().dk_paged_attention_decode(ctypes.byref(a), None) == 1


def test_misaligned_pointer_is_rejected():
    a = _args()
    a.k_cache += 2  # not aligned to head_dim / 16 = 8 bytes
    rc, _ = _plan(a)
    assert rc == 1 and "aligned" in capi.last_error()


def test_plan_without_workspace_is_single_pass():
    rc, p = _plan(_args(max_seq_len=4000))
    assert rc == 0
    assert p["split"] == 0 and p["num_partitions"] == 1 and p["partition_size"] == 4032
    assert p["path"] == capi.DK_PATH_TMA_MMA and p["launches"] == 1


def _ws(n, hq, parts, d=128):
    return (torch.zeros(n, hq, parts, d), torch.zeros(n, hq, parts), torch.zeros(n, hq, parts))


def test_plan_splits_to_fill_the_gpu():
    # batch 1, 128K context, 8 KV heads: split so the grid fills the GPU
    parts = capi.num_partitions(1, 8, 128, 16, 131072)
    rc, p = _plan(_args(n=1, hq=64, hkv=8, max_seq_len=131072, ws=_ws(1, 64, parts)))
    assert rc == 0 and p["split"] == 1 and p["launches"] == 2
    assert p["partition_size"] <= 4096 and p["partition_size"] % 64 == 0
    assert p["num_partitions"] * p["partition_size"] >= 131072
    assert p["num_ctas"] == p["num_partitions"] * 8
    # about one wave of two CTAs per SM on a 148-SM B200 (the planner's target)
    assert 2 * 148 <= p["num_ctas"] <= 2 * 148 + 8


def test_plan_respects_a_small_workspace():
    # the reference's own sizing (ceil(L / 512) partitions) leaves the planner free
    rc, p = _plan(_args(n=1, hq=64, hkv=8, max_seq_len=131072, ws=_ws(1, 64, 256)))
    assert rc == 0 and p["num_partitions"] <= 256
    # a smaller workspace grows the partitions instead
    rc, p = _plan(_args(n=1, hq=64, hkv=8, max_seq_len=131072, ws=_ws(1, 64, 10)))
    assert rc == 0 and p["num_partitions"] <= 10 and p["partition_size"] % 64 == 0


def test_plan_with_merge_counters_is_one_launch():
    ctr = torch.zeros(4 * 8, dtype=torch.int32)
    # 6 rows x 4 heads x 130 floats per (sequence, KV head): merged in the partition kernel
    rc, p = _plan(_args(max_seq_len=3000, ws=(*_ws(4, 32, 47), ctr), partition_size=512))
    assert rc == 0 and p["split"] == 1 and p["launches"] == 1
    # 47 rows (97 KB): the separate merge kernel, unless forced
    rc, p = _plan(_args(max_seq_len=3000, ws=(*_ws(4, 32, 47), ctr), partition_size=64))
    assert rc == 0 and p["split"] == 1 and p["launches"] == 2
    rc, p = _plan(_args(max_seq_len=3000, ws=(*_ws(4, 32, 47), ctr), partition_size=64,
                        flags=capi.DK_FLAG_FORCE_FUSED_MERGE))
    assert rc == 0 and p["split"] == 1 and p["launches"] == 1
    # single pass ignores the counters
    rc, p = _plan(_args(max_seq_len=3000, ws=None, merge_counters=ctr.data_ptr()))
    assert rc == 0 and p["split"] == 0 and p["launches"] == 1
    a = _args(max_seq_len=3000, ws=_ws(4, 32, 47))
    a.merge_counters = ctr.data_ptr() + 2
    assert _plan(a)[0] == 1 and "merge_counters" in capi.last_error()


def test_misaligned_workspace_is_rejected():
    a = _args(max_seq_len=3000, ws=_ws(4, 32, 47))
    a.tmp_out += 4
    assert _plan(a)[0] == 1 and "16-byte aligned" in capi.last_error()


def test_fp8_caches_plan_and_validate():
    kv8 = torch.zeros(64, 16, 8, 128, dtype=torch.uint8)
    q = torch.zeros(4, 32, 128, dtype=torch.bfloat16)
    bt = torch.zeros(4, 64, dtype=torch.int32)
    sl = torch.zeros(4, dtype=torch.int32)
    a = capi.make_args(q, kv8, kv8, bt, sl, 128**-0.5, 3000, q, _ws(4, 32, 47), 0, False, 0, 0.5, 0.25)
    assert a.kv_fp8 == 1 and a.k_scale == 0.5
    rc, p = _plan(a)
    assert rc == 0 and p["path"] == capi.DK_PATH_TMA_MMA and p["stages"] == 2 and p["partition_size"] % 128 == 0
    # e4m3 rows of 64 bytes go to the CUDA-core path
    kv64 = torch.zeros(64, 16, 8, 64, dtype=torch.uint8)
    q64 = torch.zeros(4, 32, 64, dtype=torch.bfloat16)
    rc, p = _plan(capi.make_args(q64, kv64, kv64, bt, sl, 0.125, 3000, q64, None, 0, False, 0, 1.0, 1.0))
    assert rc == 0 and p["path"] == capi.DK_PATH_SIMT
    a.v_scale = 0.0
    assert _plan(a)[0] == 1 and "k_scale and v_scale" in capi.last_error()
    a.v_scale, a.kv_fp8 = 1.0, 3
    assert _plan(a)[0] == 1 and "kv_fp8" in capi.last_error()


def test_plan_fixed_partition_size():
    rc, p = _plan(_args(max_seq_len=3000, ws=_ws(4, 32, 47), partition_size=64))
    assert rc == 0 and p["partition_size"] == 64 and p["num_partitions"] == 47


def test_plan_path_choice():
    assert _plan(_args(bs=16))[1]["path"] == capi.DK_PATH_TMA_MMA
    assert _plan(_args(bs=256))[1]["path"] == capi.DK_PATH_TMA_MMA
    assert _plan(_args(bs=8))[1]["path"] == capi.DK_PATH_TMA_MMA
    assert _plan(_args(bs=4))[1]["path"] == capi.DK_PATH_SIMT
    assert _plan(_args(bs=48))[1]["path"] == capi.DK_PATH_SIMT
    assert _plan(_args(force_simt=True))[1]["path"] == capi.DK_PATH_SIMT


def test_num_partitions_bounds():
    for n, hkv, L in [(1, 8, 131072), (64, 8, 4096), (256, 8, 32768), (4, 8, 513), (128, 1, 32768)]:
        p = capi.num_partitions(n, hkv, 128, 16, L)
        assert 1 <= p <= -(-L // 128) and p * 4096 >= L  # partitions of 128..4096 tokens
        assert capi.num_partitions(n, 0, 128, 16, L) >= p  # unknown head count sizes for the most
    assert capi.num_partitions(4, 8, 128, 16, 0) == 1
    with pytest.raises(ValueError):
        capi.num_partitions(4, 8, 96, 16, 100)


def test_empty_batch_is_a_no_op():
    a = _args(n=0)
    rc, p = _plan(a)
    assert rc == 0 and p["path"] == capi.DK_PATH_NONE
    assert capi.load().dk_paged_attention_decode(ctypes.byref(a), None) == 0


def _wide_ws(n, hq, parts, d):
    """A workspace's shape without its memory (the planner reads sizes only)."""
    z = torch.zeros(1)
    return (z.expand(n, hq, parts, d), z.expand(n, hq, parts), z.expand(n, hq, parts))


@pytest.mark.parametrize(
    "n,hq,hkv,d,bs,L,want",
    [
        (256, 64, 8, 128, 16, 32768, 4096),  # c5: many (sequence, KV head) pairs -> the byte cap
        (256, 32, 4, 128, 16, 32768, 4096),  # a rank's share of c5 at 2 GPUs (1024 pairs)
        (256, 16, 2, 128, 16, 32768, 4096),  # ... at 4 GPUs
        (256, 8, 1, 128, 16, 32768, 3520),   # ... at 8 GPUs: ~8 waves of CTAs at max_seq_len
        (64, 32, 8, 128, 16, 4096, 1024),    # c2: the 512 KB floor
        (128, 8, 1, 256, 32, 32768, 1728),   # c4 (MQA, D = 256)
    ],
)
def test_planner_partition_sizes(n, hq, hkv, d, bs, L, want):
    """The planner's choices for the measured shapes (148 SMs assumed without
    a GPU): few pairs get partitions for ~8 waves of CTAs, within
    [512 KB, 2 MB] of 16-bit K+V.  16-bit caches never fit the size on the
    device."""
    rc, p = _plan(_args(n=n, hq=hq, hkv=hkv, d=d, bs=bs, max_seq_len=L, ws=_wide_ws(n, hq, -(-L // 64), d)))
    assert rc == 0, capi.last_error()
    assert p["partition_size"] == want and p["fit_min_partition"] == 0
    assert p["num_partitions"] == -(-L // want)
    assert capi.num_partitions(n, hkv, d, bs, L) >= p["num_partitions"]


def _fp8_plan(n, hq, hkv, d, bs, L, rows, partition_size=0):
    kv8 = torch.zeros(64, bs, hkv, d, dtype=torch.uint8)
    q = torch.zeros(n, hq, d, dtype=torch.bfloat16)
    bt = torch.zeros(n, 64, dtype=torch.int32)
    sl = torch.zeros(n, dtype=torch.int32)
    a = capi.make_args(q, kv8, kv8, bt, sl, d**-0.5, L, q, _wide_ws(n, hq, rows, d), partition_size, False, 0, 0.5,
                       0.5)
    return _plan(a)


def test_fitted_partition_floor_follows_the_workspace():
    """e4m3 c4's shape: the planned 1728 tokens bound the device's fit, down
    to 512 with the workspace the library sizes (its rows: down to 512 tokens,
    plus the row passing the choice to the merge kernel).  Fewer rows raise
    the floor (the last row stays out of the partitions' reach); too few for
    any fit leave the planned size fixed; a size the caller fixes is never
    fitted; neither is a lone sequence, nor a batch with more (sequence, KV
    head) pairs than SMs."""
    n, hq, hkv, d, bs, L = 128, 8, 1, 256, 32, 32768
    rows = capi.num_partitions(n, hkv, d, bs, L)
    assert rows == L // 512 + 1
    rc, p = _fp8_plan(n, hq, hkv, d, bs, L, rows)
    assert rc == 0 and p["partition_size"] == 1728 and p["fit_min_partition"] == 512 and p["num_partitions"] == rows
    rc, p = _fp8_plan(n, hq, hkv, d, bs, L, 32)
    assert rc == 0 and p["fit_min_partition"] == 1088 and p["num_partitions"] == 32 and p["partition_size"] == 1728
    rc, p = _fp8_plan(n, hq, hkv, d, bs, L, 19)
    assert rc == 0 and p["fit_min_partition"] == 0 and p["num_partitions"] == 19
    rc, p = _fp8_plan(n, hq, hkv, d, bs, L, rows, partition_size=1024)
    assert rc == 0 and p["fit_min_partition"] == 0 and p["partition_size"] == 1024
    rc, p = _fp8_plan(1, 64, 8, 128, 16, 131072, 2048)
    assert rc == 0 and p["fit_min_partition"] == 0
    rc, p = _fp8_plan(160, 8, 1, 256, 32, L, rows)
    assert rc == 0 and p["fit_min_partition"] == 0
