"""Device-side bounds checks (SURVEY's substitute for compute-sanitizer, which is closed on
this pool): the debug build libsnnb200_check.so compiles index checks into the kernels'
global loads and stores that record SNNB_ERR_DEVICE in the device status word and skip the
access.  Tail and ragged shapes (partial pixel and channel blocks, ragged neuron counts,
partial image-layer tiles) run under it must leave the status word clear and give the same
outputs as the release build."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "triton-pass-analysis_b200")


def _run(tmp_path, name, library):
    path = str(tmp_path / f"{name}.pt")
    env = dict(os.environ)
    env.pop("SNNB_LIBRARY", None)
    if library:
        env["SNNB_LIBRARY"] = library
    subprocess.run([sys.executable, os.path.join(HERE, "bounds_cases.py"), path], env=env,
                   check=True, timeout=600)
    return torch.load(path)


def test_tail_shapes_pass_the_device_bounds_checks(tmp_path):
    check_lib = os.path.join(PKG, "libsnnb200_check.so")
    assert os.path.exists(check_lib), "build it with `make -C triton-pass-analysis_b200 check`"
    rel = _run(tmp_path, "release", None)
    chk = _run(tmp_path, "check", check_lib)
    assert int(chk["status"]) == 0, "a device-side index check failed"
    assert int(rel["status"]) == 0
    assert rel.keys() == chk.keys()
    for k in rel:
        assert torch.equal(rel[k], chk[k]), k
