"""The B200 backend of the reference expert node (constellation_b200/plugin), compiled
against the node's own headers (expert_node_v2/backend/backend_workspace_v2.h,
backend_registry_v2.h, expert_format_v2.h) and driven through them by
``tests/c_abi/plugin_driver.cc``.

* CPU: builds the backend and the driver from the reference tree here, and runs the
  status-only paths (no device: nothing initialises, uploads fail and leave the storage
  empty, a request is refused so the worker answers status 4).
* GPU: runs the driver built by ``__graft_entry__.build()`` (the reference tree is absent
  on a GPU machine): two experts uploaded through the registry's upload hook, requests of
  batch 3 / 1 / 5 in bf16 and fp16 through ``RunExpertRequest``, a replacement upload,
  malformed requests and a foreign storage; outputs against the CPU oracle (row-wise
  relative error <= 1e-2, the 16-bit output bar of the other tests).
"""
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PLUGIN = ROOT / "constellation_b200" / "plugin"
DRIVER_SRC = Path(__file__).resolve().parent / "c_abi" / "plugin_driver.cc"
PREBUILT = PLUGIN / "_build" / "plugin_driver"
H, I = 256, 128


def build_driver(out_dir: Path) -> Path:
    from oracle import refbuild

    root = refbuild.reference_root()
    if root is None:
        pytest.skip("the reference tree is not present")
    if shutil.which("g++") is None or shutil.which("make") is None:
        pytest.skip("g++ / make not installed")
    r = subprocess.run(["make", "-s", "-C", str(PLUGIN), f"REF={root}", f"OUT={out_dir}", f"DRIVER={DRIVER_SRC}",
                        "driver"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return out_dir / "plugin_driver"


def test_plugin_builds_against_reference_headers_and_refuses_without_a_device(tmp_path):
    exe = build_driver(tmp_path)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")  # the status-only paths, even on a GPU machine
    out = subprocess.run([str(exe), "cpu"], capture_output=True, text=True, timeout=120, env=env)
    assert out.returncode == 0 and "cpu-ok" in out.stdout, out.stdout + out.stderr


def _write_expert(d: Path, e: int, bundle) -> None:
    for name, arr in (("w_up", bundle.w_up), ("s_up", bundle.s_up), ("w_gate", bundle.w_gate),
                      ("s_gate", bundle.s_gate), ("w_down", bundle.w_down), ("s_down", bundle.s_down)):
        np.ascontiguousarray(arr).tofile(d / f"e{e}_{name}.bin")


@pytest.mark.gpu
def test_plugin_serves_requests_through_the_node_interfaces(tmp_path):
    import torch

    from oracle import cases, codec
    from oracle.expert import DequantExpert

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not PREBUILT.is_file():
        pytest.skip("plugin_driver was not built (the reference tree was absent at build time)")
    e0, e1 = cases.expert(9100, H, I), cases.expert(9101, H, I)
    _write_expert(tmp_path, 0, e0)
    _write_expert(tmp_path, 1, e1)
    x3 = cases.activations(9102, 3, H)
    x1 = cases.activations(9103, 1, H)
    x5 = cases.activations(9104, 5, H)
    codec.encode_bf16_rne(x3).tofile(tmp_path / "x3_bf16.bin")
    x1_16 = torch.from_numpy(x1).to(torch.float16)
    x1_16.view(torch.int16).numpy().tofile(tmp_path / "x1_fp16.bin")
    codec.encode_bf16_rne(x5).tofile(tmp_path / "x5_bf16.bin")
    out = subprocess.run([str(PREBUILT), "gpu", str(tmp_path)], capture_output=True, text=True, timeout=300)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = {ln.split()[0]: ln for ln in out.stdout.splitlines() if ln.strip()}
    for tag, batch, dt in (("req1", 3, 2), ("req2", 1, 2), ("req3", 5, 1), ("req4", 3, 2)):
        assert f"ok=1 status=0 batch={batch} hidden={H} dtype={dt} bytes={batch * H * 2}" in lines[tag], lines[tag]
    for tag in ("bad_bytes", "bad_dtype", "bad_batch", "foreign"):
        assert "ok=0" in lines[tag], lines[tag]

    def got(name, dt):
        raw = np.fromfile(tmp_path / name, dtype=np.uint16)
        return (codec.decode_bf16(raw) if dt == 2 else codec.decode_fp16(raw)).reshape(-1, H)

    def rel(a, ref):
        return float((np.abs(a - ref).max(axis=1) / np.abs(ref).max(axis=1)).max())

    x3b = codec.decode_bf16(codec.encode_bf16_rne(x3))
    x5b = codec.decode_bf16(codec.encode_bf16_rne(x5))
    x1h = x1_16.float().numpy()
    d0, d1 = DequantExpert(e0), DequantExpert(e1)
    assert rel(got("out1.bin", 2), d0.forward(x3b)) <= 1e-2
    assert rel(got("out2.bin", 2), d1.forward(x1h)) <= 1e-2
    assert rel(got("out3.bin", 1), d1.forward(x5b)) <= 1e-2
    assert rel(got("out4.bin", 2), d1.forward(x3b)) <= 1e-2  # the replaced storage serves expert 1
