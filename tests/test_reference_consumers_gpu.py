"""The reference's own consumers, unchanged, on the drop-in modules.

The drop-in promise is that the reference's communication module, its
benchmark harness and its tests run on these kernels without edits. This
test builds the merge that the integration notes describe in a temporary
directory and runs, in subprocesses on the GPU:

* the reference's in-scope module tests (tests/test_zorder_comm.py, and the
  reduce-to-dense identity of tests/test_comm_module.py:33-67) with torch's
  default device set to CUDA, since the drop-in has no CPU path;
* scripts/bench_attention_core.py and scripts/bench_prescore.py at a tiny
  configuration (their equivalence checks against the eager path included).

The merge (the same steps a maintainer follows):
1. copy the reference tree;
2. copy ``topk-tarmac_b200/src/kernels/*.py`` over its ``src/kernels/``;
3. add this build's ``src/agents/mappo.py`` as ``src/agents/tarmac_comm.py``
   and rebind ``AttentionComm`` at the end of the reference's
   ``src/agents/mappo.py``, so ``MAPPOAgent`` and every caller construct the
   kernel-backed module while the actor, critic and config stay the
   reference's;
4. put ``tarmac_b200`` (only) on the import path.

The reference tree is not part of this repository. The test looks for it in
``$TARMAC_REFERENCE_TREE`` or ``baseline/_ref/TopK-TarMAC`` and is skipped
with the reason "reference tree absent" when neither holds it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "topk-tarmac_b200"

# reference tests that pin the attention core and can run on fp32 kernels
REFERENCE_TESTS = [
    "tests/test_zorder_comm.py",
    "tests/test_comm_module.py::test_topk_at_n_minus_1_equals_dense",
    "tests/test_comm_module.py::test_topk_at_n_minus_1_equals_dense_across_n",
]

REBIND = ("\n\n# tarmac_b200 drop-in: the attention core runs on the sm_100a "
          "kernels\nfrom src.agents.tarmac_comm import AttentionComm  "
          "# noqa: E402,F401,F811\n")

CUDA_DEFAULT_PLUGIN = ('"""pytest plugin: tensors and modules the tests '
                       'create live on the GPU."""\nimport torch\n\n'
                       'torch.set_default_device("cuda")\n')


def _reference_tree() -> Path | None:
    for cand in (os.environ.get("TARMAC_REFERENCE_TREE"),
                 str(REPO / "baseline" / "_ref" / "TopK-TarMAC")):
        if cand and (Path(cand) / "src" / "kernels" /
                     "fused_topk_attention.py").exists():
            return Path(cand)
    return None


@pytest.fixture(scope="module")
def merged(tmp_path_factory):
    ref = _reference_tree()
    if ref is None:
        pytest.skip("reference tree absent")
    root = tmp_path_factory.mktemp("merged")
    tree = root / "TopK-TarMAC"
    shutil.copytree(ref, tree, ignore=shutil.ignore_patterns(
        ".git", "__pycache__", "*.png", "*.pdf"))
    for f in (PKG / "src" / "kernels").glob("*.py"):
        if f.name != "__init__.py":
            shutil.copy2(f, tree / "src" / "kernels" / f.name)
    shutil.copy2(PKG / "src" / "agents" / "mappo.py",
                 tree / "src" / "agents" / "tarmac_comm.py")
    with open(tree / "src" / "agents" / "mappo.py", "a") as fh:
        fh.write(REBIND)
    pkgs = root / "pkgs"
    pkgs.mkdir()
    (pkgs / "tarmac_b200").symlink_to(PKG / "tarmac_b200",
                                      target_is_directory=True)
    (pkgs / "tarmac_cuda_default.py").write_text(CUDA_DEFAULT_PLUGIN)
    env = dict(os.environ)
    env["PYTHONPATH"] = str(pkgs)
    env.pop("TRITON_INTERPRET", None)
    return tree, env


def _run(cmd, cwd, env, timeout=900):
    r = subprocess.run(cmd, cwd=cwd, env=env, capture_output=True, text=True,
                       timeout=timeout)
    return r.returncode, (r.stdout[-4000:] + "\n" + r.stderr[-4000:])


def test_merge_uses_the_kernel_backed_module(merged):
    tree, env = merged
    code = ("import src.agents.mappo as m, src.agents.tarmac_comm as t;"
            "assert m.AttentionComm is t.AttentionComm;"
            "import src.kernels.fused_topk_attention as f;"
            "import tarmac_b200, inspect;"
            "assert 'tarmac_b200' in inspect.getsource(f);"
            "print('merged ok')")
    rc, out = _run([sys.executable, "-c", code], tree, env)
    assert rc == 0 and "merged ok" in out, out


def test_reference_module_tests_pass_on_the_kernels(merged):
    tree, env = merged
    rc, out = _run([sys.executable, "-m", "pytest", "-q", "-p",
                    "tarmac_cuda_default", "-p", "no:cacheprovider",
                    *REFERENCE_TESTS], tree, env)
    assert rc == 0, out


def test_reference_harness_attention_core(merged, tmp_path):
    tree, env = merged
    rc, out = _run([sys.executable, "scripts/bench_attention_core.py",
                    "--device", "cuda:0", "--n-list", "48", "192",
                    "--k-list", "1", "2", "--batch-list", "16",
                    "--reps", "2", "--warmup", "1", "--runs", "1",
                    "--out", str(tmp_path / "attention_core.json")],
                   tree, env)
    assert rc == 0, out
    assert (tmp_path / "attention_core.json").exists()


def test_reference_harness_prescore(merged, tmp_path):
    tree, env = merged
    rc, out = _run([sys.executable, "scripts/bench_prescore.py",
                    "--device", "cuda:0", "--n-list", "64", "256",
                    "--k-list", "2", "--batch", "16", "--reps", "2",
                    "--warmup", "1", "--runs", "1",
                    "--out", str(tmp_path / "prescore.json")], tree, env)
    assert rc == 0, out
    assert (tmp_path / "prescore.json").exists()
