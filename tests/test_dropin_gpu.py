"""The drop-in boundary: the reference's own DiT, calibration and sampler modules (qwen_image21.py, calibrate.py,
sampling.py, unmodified) run on this build's tfimage API (linear.py, kernels.py, ext.py, _lib.py, store.py), the
way a maintainer installs it: the reference package with this build's modules in place of its TensorFold-backed
ones. The reference checkout is looked up in $TFIMAGE_REFERENCE (a directory holding the reference's ``tfimage``
package) or in baseline/_ref (the reference installed by pip); without it the test is skipped.

The assembled package runs in a child interpreter (tests/_dropin_child.py): a reduced QwenImage21 (2 blocks,
dim 256, 2 heads x 128, MLP 512) with make("nvfp4") linears, the reference's calibrate() (dynamic input scales and the
unfused MLP fallback, then static scales and the fused MLP), two forward() calls through the kept-prefix path, a
store.save / store.load round trip, and the same reference model on oracle-backed linears and fusions as the
checker (with the reference's fp32 GEMM sums, and once more with exact sums)."""

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "qwen-image21-tensorfold-rtx_b200" / "tfimage"
REFERENCE_MODULES = ("__init__.py", "qwen_image21.py", "calibrate.py", "sampling.py")
OUR_MODULES = ("linear.py", "kernels.py", "ext.py", "_lib.py", "store.py", "gguf_load.py")


def _reference_package():
    base = os.environ.get("TFIMAGE_REFERENCE") or str(ROOT / "baseline" / "_ref")
    p = Path(base) / "tfimage"
    return p if all((p / f).is_file() for f in REFERENCE_MODULES) else None


def test_reference_dit_runs_unchanged_on_this_api(dev, tmp_path):
    ref = _reference_package()
    if ref is None:
        pytest.skip("the reference's tfimage package is not installed ($TFIMAGE_REFERENCE or baseline/_ref)")
    pkg = tmp_path / "pkg" / "tfimage"
    pkg.mkdir(parents=True)
    for f in REFERENCE_MODULES:
        shutil.copyfile(ref / f, pkg / f)
    for f in OUR_MODULES:
        shutil.copyfile(PKG / f, pkg / f)
    out = tmp_path / "result.json"
    env = dict(os.environ, TFIMAGE_EXT_DIR=str(PKG))        # libtfb.so from this repository (ext.use_prebuilt)
    proc = subprocess.run([sys.executable, str(Path(__file__).parent / "_dropin_child.py"), str(tmp_path / "pkg"),
                           str(ROOT), str(out), str(tmp_path)], env=env, capture_output=True, text=True, timeout=900)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    r = json.loads(out.read_text())
    print(r)
    assert r["kinds"] == ["Nvfp4Linear"]                     # make("nvfp4") gave this build's NVFP4 layers
    assert r["dynamic_before"] and r["static_after"]         # calibrate(): set_act(None), amax, set_act(margin * amax)
    assert r["fused_mlp"]                                    # static layers take the fused gate/up + down pair
    assert r["prefix_reused"] and r["repeat_equal"] and r["finite"]
    assert r["shape"] == [1, 64, 8, 8]
    assert r["store_equal"] and r["store_cfg"]               # store.save -> store.load gives the same model
    # against the oracle-backed reference model with exact GEMM sums: 2e-3 (measured: bit-identical); against the
    # reference's fp32 sums: 2e-3, or twice the checker's own fp32-vs-exact spread where that is larger (each block
    # chains several NVFP4 requantizations, which turn last-bit differences into code / block-scale changes)
    assert r["rel_l2_vs_exact_sums"] <= 2e-3, r
    assert r["rel_l2"] <= max(2e-3, 2.0 * r["checker_fp32_vs_exact_sums"]), r
