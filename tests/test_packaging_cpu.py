"""CPU: DecodeKernels' import path (``import decode_kernels as dk``) and the
vLLM plugin registration of the installed package.

* ``decode_kernels`` exports the reference's attention names
  (``decode_kernels/__init__.py:7-27``, ``ops.py:14-116``) as this library's
  objects, with the reference's signatures.
* ``pip install`` of the repository (into a temporary prefix) registers the
  ``vllm.general_plugins`` entry point the reference declares
  (``pyproject.toml:22-23``), and the entry point loads from the installed
  copy and does nothing while ``DECODE_KERNELS_VLLM`` is unset.
"""

import importlib.metadata
import inspect
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_decode_kernels_import_path_matches_the_reference_names():
    import decode_kernels as dk
    import decodekernels_b200 as impl
    from decode_kernels import ops

    for name in ("PARTITION_SIZE", "alloc_workspace", "is_available", "paged_attention_decode"):
        assert getattr(dk, name) is getattr(impl, name), name
    assert (ops.PARTITION_SIZE, ops.MAX_GQA_GROUP, ops.SUPPORTED_HEAD_DIMS) == (512, 8, (64, 128, 256))
    assert ops.num_partitions(513) == 2  # the reference's ceil(L / 512)
    params = list(inspect.signature(dk.paged_attention_decode).parameters)
    assert params[:9] == ["q", "k_cache", "v_cache", "block_tables", "seq_lens", "scale", "max_seq_len", "out",
                          "workspace"]
    params = list(inspect.signature(dk.alloc_workspace).parameters)
    assert params[:5] == ["num_seqs", "num_q_heads", "head_dim", "max_seq_len", "device"]
    from decode_kernels import testing, vllm_patch, vllm_plugin

    assert callable(vllm_plugin.register) and callable(vllm_patch.apply) and callable(testing.make_paged_kv)


def test_installed_package_registers_the_vllm_plugin(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    shutil.copy(ROOT / "pyproject.toml", src)
    for pkg in ("decodekernels_b200", "decode_kernels"):
        shutil.copytree(ROOT / pkg, src / pkg, ignore=shutil.ignore_patterns("__pycache__"))
    site = tmp_path / "site"
    r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                        "--quiet", "--target", str(site), str(src)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    eps = [ep for d in importlib.metadata.distributions(path=[str(site)]) for ep in d.entry_points
           if ep.group == "vllm.general_plugins"]
    assert [(ep.name, ep.value) for ep in eps] == [("decode_kernels", "decode_kernels.vllm_plugin:register")]

    code = ("import importlib.metadata as m\n"
            "ep = [e for e in m.entry_points(group='vllm.general_plugins') if e.name == 'decode_kernels'][0]\n"
            "register = ep.load()\n"
            "import decode_kernels, decodekernels_b200\n"
            "assert register() is None\n"
            "print(decode_kernels.__file__)\n"
            "print(decodekernels_b200.__file__)\n")
    env = {k: v for k, v in os.environ.items() if k not in ("PYTHONPATH", "DECODE_KERNELS_VLLM")}
    env["PYTHONPATH"] = str(site)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd=tmp_path,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    files = r.stdout.split()
    assert len(files) == 2 and all(f.startswith(str(site)) for f in files), r.stdout
