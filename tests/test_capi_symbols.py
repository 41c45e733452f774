"""The C-ABI library loads on a machine without a GPU and exports every declared symbol."""
import ctypes
import re
import subprocess
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "constellation_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|void|int32_t|const char\*)\s+\**(cst_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert "cst_create" in syms and "cst_moe_layer" in syms and "cst_expert_forward" in syms
    assert len(syms) >= 15


def test_library_exports_every_declared_symbol():
    from constellation_b200 import _lib

    lib = _lib.lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s(cst_\w+)$", out, re.M))
    for s in declared_symbols():
        assert s in exported, s
        assert isinstance(getattr(lib, s), ctypes._CFuncPtr)
    assert set(_lib.EXPORTED) == set(declared_symbols())


def test_abi_version_and_last_error_without_gpu():
    from constellation_b200 import _lib

    assert _lib.lib.cst_abi_version() == 100
    assert isinstance(_lib.last_error(), str)


def test_invalid_config_is_rejected_before_touching_a_device():
    from constellation_b200 import _lib

    cfg = _lib.CstConfig(hidden_dim=100, inter_dim=128, n_routed_experts=256, n_group=8, topk_group=4, top_k=8,
                         norm_topk_prob=1, routed_scaling_factor=2.5, block_size=128, n_slots=1, max_tokens=4,
                         max_rows=0)
    h = ctypes.c_void_p()
    rc = _lib.lib.cst_create(0, ctypes.byref(cfg), ctypes.byref(h))
    assert rc == _lib.CST_ERR_INVALID_ARG
    assert "multiples of 128" in _lib.last_error()
    cfg.hidden_dim = 256
    cfg.block_size = 64
    assert _lib.lib.cst_create(0, ctypes.byref(cfg), ctypes.byref(h)) == _lib.CST_ERR_INVALID_ARG
    assert h.value is None


def test_empty_batch_needs_no_device_or_pointers():
    """T = 0 returns CST_OK once the scalar arguments are valid, with NULL data pointers
    (a zero-size device tensor has one); invalid scalars are still rejected."""
    from constellation_b200 import _lib

    L = _lib.lib
    assert L.cst_rmsnorm(None, 2, 0, 256, None, 1e-6, None, 2, None) == _lib.CST_OK
    assert L.cst_rmsnorm(None, 2, 0, 12, None, 1e-6, None, 2, None) == _lib.CST_ERR_INVALID_ARG
    assert L.cst_rmsnorm(None, 2, 1, 256, None, 1e-6, None, 2, None) == _lib.CST_ERR_INVALID_ARG
    route = (256, None, None, None, 16, 4, 2, 4, 1, 2.5, None, None, None)
    assert L.cst_route_noalloc(None, 2, 0, *route) == _lib.CST_OK
    assert L.cst_route_noalloc(None, 2, -1, *route) == _lib.CST_ERR_INVALID_ARG
    assert L.cst_route_noalloc(None, 2, 1, *route) == _lib.CST_ERR_INVALID_ARG
    assert "null pointer" in _lib.last_error()


def test_product_has_no_oracle_dependency():
    """The shipped package never imports the oracle (it is test infrastructure)."""
    pkg = REPO / "constellation_b200"
    for p in pkg.rglob("*.py"):
        src = p.read_text()
        assert not re.search(r"^\s*(from|import)\s+oracle\b", src, re.M), p


def test_peer_set_layout_matches_the_header():
    """cst_peer_set (include/constellation_b200.h) as ctypes sees it: four int32, then
    CST_MAX_PEERS receive pointers, CST_MAX_PEERS counter pointers, epoch, reserved."""
    import ctypes

    from constellation_b200._lib import CST_MAX_PEERS, CstIpcHandle, CstPeerSet

    P = ctypes.sizeof(ctypes.c_void_p)
    assert CstPeerSet.recv.offset == 16
    assert CstPeerSet.flags.offset == 16 + CST_MAX_PEERS * P
    assert CstPeerSet.epoch.offset == 16 + 2 * CST_MAX_PEERS * P
    assert CstPeerSet.x_offset.offset == 16 + (2 * CST_MAX_PEERS + 2) * P
    assert CstPeerSet.gather_epoch.offset == 16 + (2 * CST_MAX_PEERS + 2) * P + 8
    assert CstPeerSet.presence_offset.offset == 16 + (2 * CST_MAX_PEERS + 3) * P + 8
    assert ctypes.sizeof(CstPeerSet) == 16 + (2 * CST_MAX_PEERS + 3) * P + 16
    assert ctypes.sizeof(CstIpcHandle) == 64
    hdr = (Path(__file__).resolve().parents[1] / "include" / "constellation_b200.h").read_text()
    assert f"#define CST_MAX_PEERS {CST_MAX_PEERS}" in hdr
