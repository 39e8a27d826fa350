"""Write the golden vectors that pin the CPU oracle and the CUDA path.

Run in a container that has the DecodeKernels reference tree mounted
(``DK_REFERENCE_DIR``, else a ``reference`` directory beside this
repository's checkout):

    python tests/golden/make_golden.py

It imports the reference's own ``decode_kernels/reference.py`` and
``decode_kernels/testing.py`` straight from that tree (under aliased module
names, without installing or copying them), builds each case below with the
reference's ``make_paged_kv`` and a seeded query batch, runs the reference's
``paged_attention_reference`` (dense) and ``split_k_attention_reference``
(flash-decoding merge), and writes:

* ``tests/golden/cases.json`` -- per case: the arguments, sha256 digests of
  every input tensor (so a replay can prove it rebuilt the same inputs), and
  the partition sizes used;
* ``tests/golden/<name>.npz`` -- the reference outputs (float32 arrays;
  half-precision dense outputs are stored as their exact float32 values).

The cases follow the reference's own tests (``tests/test_reference.py`` and
``tests/test_kernels.py``) and the CPU-runnable config of the benchmark spec.
Nothing at test time reads the reference tree: tests replay the cases with
``decodekernels_b200.testing.make_paged_kv`` and compare digests.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ["DK_REFERENCE_DIR"]) if os.environ.get("DK_REFERENCE_DIR") else \
    HERE.parent.parent.parent / "reference"

sys.path.insert(0, str(HERE.parent.parent))
from decodekernels_b200.testing import tensor_digest  # noqa: E402


def _load(alias: str, path: Path):
    spec = importlib.util.spec_from_file_location(alias, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[alias] = mod
    spec.loader.exec_module(mod)
    return mod


DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _case(name, seq_lens, num_kv_heads, group, head_dim, block_size=16, dtype="float32", layout="nhd",
          extra_blocks=3, seed=0, q_seed=1, scale=None, partitions=(512,)):
    return dict(name=name, seq_lens=list(seq_lens), num_kv_heads=num_kv_heads, num_q_heads=num_kv_heads * group,
                head_dim=head_dim, block_size=block_size, dtype=dtype, layout=layout, extra_blocks=extra_blocks,
                seed=seed, q_seed=q_seed, scale=scale, partitions=list(partitions))


SPLIT_LENS = [1, 7, 63, 64, 65, 511, 512, 513, 1300]  # tests/test_reference.py:34
CASES = [
    # split-K merge == dense across partition boundaries (tests/test_reference.py:30-42)
    _case("merge_d64_g1", SPLIT_LENS, 2, 1, 64, partitions=(64, 512)),
    _case("merge_d64_g4", SPLIT_LENS, 2, 4, 64, partitions=(64, 512)),
    _case("merge_d128_g8", SPLIT_LENS, 2, 8, 128, partitions=(64, 512)),
    # paged gather == contiguous attention for several block sizes (:45-63)
    _case("gather_bs1", [5, 33, 100], 2, 4, 64, block_size=1),
    _case("gather_bs16", [5, 33, 100], 2, 4, 64, block_size=16),
    _case("gather_bs32", [5, 33, 100], 2, 4, 64, block_size=32),
    # strided FlashInfer-HND and vLLM-interleaved views (:66-79)
    _case("strided_hnd", [3, 40, 129], 2, 4, 64, layout="hnd"),
    _case("strided_vllm", [3, 40, 129], 2, 4, 64, layout="vllm"),
    # empty sequence gives zeros, split with a tiny partition (:89-95)
    _case("empty_fp32", [0, 10], 1, 1, 64, partitions=(4, 512)),
    # benchmark config c1 (CPU-runnable reference check): bf16, NHD, 160-block pool
    _case("c1", [1, 511, 512, 513], 8, 4, 128, dtype="bfloat16", extra_blocks=160 - 98, partitions=(512, 64)),
    # half-precision cases shaped like the reference's GPU tests (tests/test_kernels.py:36-98)
    _case("short_f16_d128_g4_bs16", [1, 2, 17, 100, 255, 512], 2, 4, 128, dtype="float16"),
    _case("short_bf16_d256_g8_bs32", [1, 2, 17, 100, 255, 512], 2, 8, 256, block_size=32, dtype="bfloat16"),
    _case("short_bf16_d64_g1_bs16", [1, 2, 17, 100, 255, 512], 2, 1, 64, dtype="bfloat16"),
    _case("split_bf16_d128_g8", [1, 511, 512, 513, 1024, 1025, 3000, 8192], 2, 8, 128, dtype="bfloat16",
          partitions=(512, 256)),
    _case("split_f16_d64_g1", [1, 511, 512, 513, 1024, 1025, 3000, 8192], 2, 1, 64, dtype="float16"),
    _case("strided_hnd_f16", [700, 2000], 2, 4, 128, dtype="float16", layout="hnd"),
    _case("strided_vllm_f16", [700, 2000], 2, 4, 128, dtype="float16", layout="vllm"),
    _case("empty_f16", [0, 50, 0, 2000], 2, 2, 64, dtype="float16"),
    _case("scale_bf16", [64, 900], 1, 4, 128, dtype="bfloat16", scale=0.05),
]


def main() -> None:
    ref = _load("dk_reference_oracle", REF / "decode_kernels" / "reference.py")
    fixtures = _load("dk_reference_testing", REF / "decode_kernels" / "testing.py")
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    meta = []
    for c in CASES:
        dtype = DT[c["dtype"]]
        kv = fixtures.make_paged_kv(c["seq_lens"], c["num_kv_heads"], c["head_dim"], c["block_size"], dtype, "cpu",
                                    layout=c["layout"], extra_blocks=c["extra_blocks"], seed=c["seed"])
        g = torch.Generator().manual_seed(c["q_seed"])
        q = torch.randn(len(c["seq_lens"]), c["num_q_heads"], c["head_dim"], generator=g, dtype=dtype)
        args = (q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
        arrays = {"dense": ref.paged_attention_reference(*args, scale=c["scale"]).float().numpy()}
        for ps in c["partitions"]:
            arrays[f"split_{ps}"] = ref.split_k_attention_reference(*args, scale=c["scale"], partition_size=ps).numpy()
        np.savez_compressed(HERE / f"{c['name']}.npz", **arrays)
        entry = dict(c)
        entry["digests"] = {
            "k_cache": tensor_digest(kv.k_cache),
            "v_cache": tensor_digest(kv.v_cache),
            "block_tables": tensor_digest(kv.block_tables),
            "seq_lens": tensor_digest(kv.seq_lens),
            "q": tensor_digest(q),
        }
        entry["k_strides"] = list(kv.k_cache.stride())
        meta.append(entry)
        print(f"{c['name']:<28} dense {arrays['dense'].shape} max|o|={np.abs(arrays['dense']).max():.3f}")
    (HERE / "cases.json").write_text(json.dumps({"reference": "JayaChandraDadi/DecodeKernels", "cases": meta},
                                                indent=1) + "\n")


if __name__ == "__main__":
    main()
