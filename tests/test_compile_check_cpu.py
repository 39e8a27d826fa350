"""CPU: the zero-spill compile check.  Every kernel instance of libdk_b200.so,
compiled for sm_100a as the library is, must spill nothing and keep no local
stack, as ptxas reports with -v (DecodeKernels makes the same check per
architecture: tools/compile_check.sh:17-40).  A spill on the decode's hot
loop turns register traffic into local-memory traffic on the HBM-bound path."""

import shutil
from pathlib import Path

import pytest

from decodekernels_b200 import build

pytestmark = pytest.mark.skipif(shutil.which(build._nvcc()) is None and not Path(build._nvcc()).exists(),
                                reason="needs nvcc")


@pytest.fixture(scope="module")
def report():
    return build.ptxas_report()


def test_every_instance_was_reported(report):
    names = [k["name"] for k in report]
    # 16-bit and e4m3 TMA partition kernels (dense grid, and compact grids of
    # two lane capacities), CUDA-core partition kernels, merges, exchange,
    # gather and cache-write kernels
    assert sum("paged_decode_tma_kernel" in n for n in names) == 30
    assert sum("paged_decode_simt_kernel" in n for n in names) == 12
    assert len(report) >= 69
    assert all(k["registers"] is not None and k["spill_stores"] is not None for k in report)


def test_no_instance_spills(report):
    bad = [f"{k['name']}: {k['registers']} registers, {k['stack_bytes']} B stack, {k['spill_stores']} B spill stores, "
           f"{k['spill_loads']} B spill loads" for k in report
           if k["spill_stores"] or k["spill_loads"] or k["stack_bytes"]]
    assert not bad, "\n".join(bad)


def test_partition_kernels_fit_their_planned_residency(report):
    # The planner's occupancy assumptions: at head_dim 64 six CTAs per SM (the
    # ring's limit), at 128 and 256 three, and four for e4m3 caches at 256
    # (their one-slice tiles' 33 KB ring leaves registers as the limit); a CTA
    # has WARPS consumer warps and a producer warp (WARPS is the 4th template
    # argument, the e4m3 flag the 5th).
    ctas = {64: 6, 128: 3, 256: 3}
    for k in report:
        if "paged_decode_tma_kernel<" not in k["name"]:
            continue
        args = [a.strip() for a in k["name"].split("paged_decode_tma_kernel<")[1].split(">")[0].split(",")]
        d, warps, fp8 = int(args[1]), int(args[3]), args[4] in ("true", "1")
        want = 4 if fp8 and d == 256 else ctas[d]
        assert k["registers"] * (warps + 1) * 32 * want <= 65536, k
