"""Per-device context of the B200 MoE path: torch-facing wrapper over the C ABI.

One ``ExpertContext`` owns one ``cst_ctx``: the expert arena of one device (its resident
experts in the kernels' fragment-major layout, see ``csrc/layout.cuh``) and the per-call
workspace.  Tensors are passed by device pointer; every call is enqueued on the current
torch CUDA stream of the context's device and nothing synchronises.  PyTorch supplies
device memory, streams and (under expert parallelism) ``torch.distributed``; all the
arithmetic of the path runs in the library's sm_100a kernels.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import CST_DTYPE_BF16, CST_DTYPE_FP16, CST_DTYPE_FP32, check

_DT = {torch.float16: CST_DTYPE_FP16, torch.bfloat16: CST_DTYPE_BF16, torch.float32: CST_DTYPE_FP32}
_DT_INV = {v: k for k, v in _DT.items()}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported activation dtype {dt}; expected float16, bfloat16 or float32") from None


@dataclass
class MoEConfig:
    """Layer geometry + router hyper-parameters (DeepSeek-V3 defaults, the benchmark's config 0)."""

    hidden_size: int = 7168
    moe_intermediate_size: int = 2048
    n_routed_experts: int = 256
    n_group: int = 8
    topk_group: int = 4
    num_experts_per_tok: int = 8
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 2.5
    block_size: int = 128
    scoring_func: str = "sigmoid"
    topk_method: str = "noaux_tc"

    def __post_init__(self):
        # the kernels implement this router only (route_token_real's own checks,
        # server/moe_layer_runtime.py:249-252)
        if self.scoring_func != "sigmoid":
            raise RuntimeError(f"unsupported scoring_func={self.scoring_func}")
        if self.topk_method != "noaux_tc":
            raise RuntimeError(f"unsupported topk_method={self.topk_method}")

    @classmethod
    def from_router_config(cls, rc: dict, inter: int) -> "MoEConfig":
        return cls(hidden_size=int(rc["hidden_size"]), moe_intermediate_size=int(inter),
                   n_routed_experts=int(rc["n_routed_experts"]), n_group=int(rc["n_group"]),
                   topk_group=int(rc["topk_group"]), num_experts_per_tok=int(rc["top_k"]),
                   norm_topk_prob=bool(rc["norm_topk_prob"]),
                   routed_scaling_factor=float(rc["routed_scaling_factor"]),
                   scoring_func=str(rc.get("scoring_func", "sigmoid")),
                   topk_method=str(rc.get("topk_method", "noaux_tc")))


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def rms_norm(x: torch.Tensor, weight: torch.Tensor | None = None, eps: float = 1e-6, *,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """``torch.nn.functional.rms_norm(x, (H,), weight, eps)`` on ``x [T, H]`` (``cst_rmsnorm``:
    fp32 math, one rounding); the prenorm before each sparse FFN
    (server/full_model_runtime.py:271-276).  ``weight`` is fp32 ``[H]`` or None."""
    if not isinstance(x, torch.Tensor) or x.dim() != 2 or not x.is_cuda:
        raise TypeError("rms_norm expects a 2-D CUDA tensor")
    x = x.contiguous()
    if weight is not None:
        if weight.dtype != torch.float32 or weight.shape != (x.shape[1],) or weight.device != x.device:
            raise RuntimeError("weight must be fp32 [H] on the device of x")
        weight = weight.contiguous()
    if out is None:
        out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        check(_lib.lib.cst_rmsnorm(x.data_ptr(), dtype_code(x.dtype), x.shape[0], x.shape[1], _ptr(weight),
                                   ctypes.c_float(eps), out.data_ptr(), dtype_code(out.dtype), _stream(x.device)))
    return out


class ExpertContext:
    """Expert arena + workspace of one CUDA device (``cst_create``)."""

    def __init__(self, device, cfg: MoEConfig, *, n_slots: int, max_tokens: int, max_rows: int = 0):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError(f"ExpertContext needs a CUDA device, got {self.device}")
        self.cfg = cfg
        self.n_slots = int(n_slots)
        self.max_tokens = int(max_tokens)
        c = _lib.CstConfig(
            hidden_dim=cfg.hidden_size, inter_dim=cfg.moe_intermediate_size,
            n_routed_experts=cfg.n_routed_experts, n_group=cfg.n_group, topk_group=cfg.topk_group,
            top_k=cfg.num_experts_per_tok, norm_topk_prob=int(bool(cfg.norm_topk_prob)),
            routed_scaling_factor=float(cfg.routed_scaling_factor), block_size=cfg.block_size,
            n_slots=self.n_slots, max_tokens=self.max_tokens, max_rows=int(max_rows))
        h = ctypes.c_void_p()
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", idx)
        torch.cuda.init()
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_create(idx, ctypes.byref(c), ctypes.byref(h)))
        self._h = h
        self.max_rows = int(max_rows) if max_rows else self.max_tokens * (cfg.num_experts_per_tok + 1)

    # -- lifecycle ---------------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.lib.cst_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        if not self._h.value:
            raise RuntimeError("ExpertContext is closed")
        return self._h

    def info(self) -> dict:
        out = (ctypes.c_int64 * 8)()
        n = _lib.lib.cst_ctx_info(self.handle, out, 8)
        keys = ["arena_bytes", "slot_bytes", "workspace_bytes", "num_sms", "resident_experts",
                "shared_slot"]
        return dict(zip(keys[:n], list(out)[:n]))

    # -- residency (BackendRegistryEntryV2 upload_expert / free_expert_weights) ----------
    def upload_expert(self, slot: int, expert_id: int, w_up, w_up_scale, w_gate, w_gate_scale,
                      w_down, w_down_scale) -> None:
        """Upload one expert in the reference format; ``expert_id = -1`` = shared expert."""
        def prep(t, dt):
            t = torch.as_tensor(t)
            if t.dtype == torch.float8_e4m3fn:
                t = t.view(torch.uint8)
            if t.dtype != dt:
                raise TypeError(f"expected {dt}, got {t.dtype}")
            return t.contiguous()

        wu, wg, wd = prep(w_up, torch.uint8), prep(w_gate, torch.uint8), prep(w_down, torch.uint8)
        su, sg, sd = (prep(s, torch.float32) for s in (w_up_scale, w_gate_scale, w_down_scale))
        if wu.dim() != 2 or wg.shape != wu.shape or wd.shape != (wu.shape[1], wu.shape[0]):
            raise RuntimeError(f"inconsistent expert shapes up={tuple(wu.shape)} gate={tuple(wg.shape)} "
                               f"down={tuple(wd.shape)}")
        b = self.cfg.block_size
        for w, s in ((wu, su), (wg, sg), (wd, sd)):
            want = ((w.shape[0] + b - 1) // b, (w.shape[1] + b - 1) // b)
            if tuple(s.shape) != want:
                raise RuntimeError(f"scale shape {tuple(s.shape)} != {want}")
        if wu.is_cuda:
            wu, wg, wd, su, sg, sd = (t.to(self.device) for t in (wu, wg, wd, su, sg, sd))
        ew = _lib.CstExpertWeights(wu.data_ptr(), su.data_ptr(), wg.data_ptr(), sg.data_ptr(), wd.data_ptr(),
                                   sd.data_ptr(), int(wu.shape[0]), int(wu.shape[1]), b, b)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_upload_expert(self.handle, int(slot), int(expert_id), ctypes.byref(ew),
                                             _stream(self.device)))

    def upload_bundle(self, slot: int, expert_id: int, e) -> None:
        """Upload an object with the six ``w_up/s_up/...`` fields (reference bundle order)."""
        self.upload_expert(slot, expert_id, e.w_up, e.s_up, e.w_gate, e.s_gate, e.w_down, e.s_down)

    def free_expert(self, slot: int) -> None:
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_free_expert(self.handle, int(slot)))

    def find_slot(self, expert_id: int) -> int:
        return int(_lib.lib.cst_find_slot(self.handle, int(expert_id)))

    def set_own_tokens_only(self, expert_id: int, flag: bool = True) -> None:
        """Serve resident expert ``expert_id`` for this rank's own tokens only (a replicated
        hot expert under expert parallelism; ``cst_set_expert_own_tokens_only``)."""
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_set_expert_own_tokens_only(self.handle, int(expert_id), int(bool(flag))))

    def find_shared_slot(self) -> int:
        """Arena slot of the shared expert (raises when none is resident)."""
        s = int(self.info().get("shared_slot", -1))
        if s < 0:
            raise RuntimeError("no shared expert is resident in this context")
        return s

    def set_shared_slot(self, slot: int) -> None:
        check(_lib.lib.cst_set_shared_slot(self.handle, int(slot)))

    def set_gemm_mode(self, mode: str) -> None:
        """Grouped-kernel shape: "auto" (prefill kernels from 32 rows per expert on),
        "decode" (16-row groups, 3 activation terms) or "prefill" (128-row groups, 2 terms)."""
        codes = {"auto": _lib.CST_GEMM_AUTO, "decode": _lib.CST_GEMM_DECODE, "prefill": _lib.CST_GEMM_PREFILL}
        if mode not in codes:
            raise ValueError(f"gemm mode must be one of {sorted(codes)}, got {mode!r}")
        check(_lib.lib.cst_set_gemm_mode(self.handle, codes[mode]))

    # -- hot path ---------------------------------------------------------------------
    def _check_x(self, x: torch.Tensor) -> torch.Tensor:
        if not isinstance(x, torch.Tensor):
            raise TypeError(f"hidden must be torch.Tensor, got {type(x).__name__}")
        if x.device != self.device:
            raise RuntimeError(f"hidden device mismatch: hidden={x.device} context={self.device}")
        if x.dim() != 2 or x.shape[1] != self.cfg.hidden_size:
            raise RuntimeError(f"hidden must be [T, {self.cfg.hidden_size}], got {tuple(x.shape)}")
        dtype_code(x.dtype)
        return x.contiguous()

    def route(self, x: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor, *,
              resident: torch.Tensor | None = None, top_k: int | None = None,
              return_aux: bool = False):
        x = self._check_x(x)
        T = x.shape[0]
        k = int(top_k or self.cfg.num_experts_per_tok)
        idx = torch.empty((T, k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, k), dtype=torch.float32, device=self.device)
        logits = gs = None
        if return_aux:
            logits = torch.empty((T, self.cfg.n_routed_experts), dtype=torch.float32, device=self.device)
            gs = torch.empty((T, self.cfg.n_group), dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_route(self.handle, x.data_ptr(), dtype_code(x.dtype), T, gate_weight.data_ptr(),
                                     bias.data_ptr(), _ptr(resident), k, idx.data_ptr(), w.data_ptr(),
                                     _ptr(logits), _ptr(gs), _stream(self.device)))
        if return_aux:
            return idx, w, logits, gs
        return idx, w

    def moe_routed(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_weight: torch.Tensor, *,
                   add_shared: bool = False, out_dtype: torch.dtype | None = None, out=None):
        x = self._check_x(x)
        T = x.shape[0]
        topk_idx = topk_idx.to(device=self.device, dtype=torch.int32).contiguous()
        topk_weight = topk_weight.to(device=self.device, dtype=torch.float32).contiguous()
        od = out_dtype or x.dtype
        if out is None:
            out = torch.empty((T, self.cfg.hidden_size), dtype=od, device=self.device)
        flags = _lib.CST_FLAG_ADD_SHARED if add_shared else 0
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_moe_routed(self.handle, x.data_ptr(), dtype_code(x.dtype), T, topk_idx.data_ptr(),
                                          topk_weight.data_ptr(), int(topk_idx.shape[1]), flags, out.data_ptr(),
                                          dtype_code(out.dtype), _stream(self.device)))
        return out

    def moe_routed_range(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_weight: torch.Tensor,
                         shared_begin: int, shared_end: int, *, out_dtype: torch.dtype = torch.float32,
                         out: torch.Tensor | None = None):
        """Routed rows of every token + the shared expert on tokens [begin, end) (EP form)."""
        x = self._check_x(x)
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.cfg.hidden_size), dtype=out_dtype, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_moe_routed_range(self.handle, x.data_ptr(), dtype_code(x.dtype), T, topk_idx.data_ptr(),
                                                topk_weight.data_ptr(), int(topk_idx.shape[1]), int(shared_begin),
                                                int(shared_end), out.data_ptr(), dtype_code(out.dtype),
                                                _stream(self.device)))
        return out

    def moe_routed_push(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_weight: torch.Tensor, peers) -> None:
        """Expert-parallel form with the combine pushed to the token owners
        (``cst_moe_routed_push``): ``x`` holds all ``world * tl`` gathered tokens; ``peers``
        is a ``CstPeerSet`` (``constellation_b200.p2p.PeerExchange.peer_set``)."""
        x = self._check_x(x)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_moe_routed_push(self.handle, x.data_ptr(), dtype_code(x.dtype), topk_idx.data_ptr(),
                                               topk_weight.data_ptr(), int(topk_idx.shape[1]), ctypes.byref(peers),
                                               _stream(self.device)))

    def gather_rows(self, x_local: torch.Tensor, peers) -> None:
        """The all-gather over peer memory (``cst_gather_rows``): this rank's ``[tl, H]``
        rows into every rank's gathered rows, then a bounded wait for all ranks' rows here."""
        x_local = self._check_x(x_local)
        if x_local.shape[0] != peers.tl:
            raise RuntimeError(f"x_local has {x_local.shape[0]} rows, the exchange {peers.tl}")
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_gather_rows(self.handle, ctypes.byref(peers), x_local.data_ptr(),
                                           dtype_code(x_local.dtype), _stream(self.device)))

    def reduce_pushed(self, peers, *, residual: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
                      out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's ``tl`` tokens: the ranks' pushed partials in rank order (+ residual),
        cast once (``cst_reduce_pushed``)."""
        if out is None:
            out = torch.empty((peers.tl, self.cfg.hidden_size), dtype=out_dtype, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_reduce_pushed(self.handle, ctypes.byref(peers), _ptr(residual),
                                             dtype_code(residual.dtype) if residual is not None else 0,
                                             out.data_ptr(), dtype_code(out.dtype), _stream(self.device)))
        return out

    def cast_extra(self, extra: torch.Tensor, *, residual: torch.Tensor | None = None,
                   out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
        """``out = extra (+ residual)`` cast once (``cst_combine_rows`` with no rows)."""
        T = extra.shape[0]
        if out is None:
            out = torch.empty((T, self.cfg.hidden_size), dtype=out_dtype, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_combine_rows(self.handle, None, 0, None, 0, T, extra.data_ptr(), _ptr(residual),
                                            dtype_code(residual.dtype) if residual is not None else 0,
                                            out.data_ptr(), dtype_code(out.dtype), _stream(self.device)))
        return out

    def moe_layer(self, x: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor, *,
                  resident: torch.Tensor | None = None, top_k: int | None = None, add_shared: bool = True,
                  residual: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                  out: torch.Tensor | None = None, return_routes: bool = False):
        x = self._check_x(x)
        T = x.shape[0]
        k = int(top_k or self.cfg.num_experts_per_tok)
        od = out_dtype or x.dtype
        if out is None:
            out = torch.empty((T, self.cfg.hidden_size), dtype=od, device=self.device)
        idx = w = None
        if return_routes:
            idx = torch.empty((T, k), dtype=torch.int32, device=self.device)
            w = torch.empty((T, k), dtype=torch.float32, device=self.device)
        if residual is not None:
            if residual.dtype != x.dtype or residual.shape != x.shape:
                raise RuntimeError("residual must match hidden in shape and dtype")
            residual = residual.contiguous()
        flags = _lib.CST_FLAG_ADD_SHARED if add_shared else 0
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_moe_layer(self.handle, x.data_ptr(), dtype_code(x.dtype), T, gate_weight.data_ptr(),
                                         bias.data_ptr(), _ptr(resident), k, flags, _ptr(residual), out.data_ptr(),
                                         dtype_code(out.dtype), _ptr(idx), _ptr(w), _stream(self.device)))
        if return_routes:
            return out, idx, w
        return out

    def grouped_ffn(self, x_rows: torch.Tensor, row_slot: torch.Tensor, row_weight: torch.Tensor | None = None,
                    *, out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None):
        x_rows = self._check_x(x_rows)
        R = x_rows.shape[0]
        row_slot = row_slot.to(device=self.device, dtype=torch.int32).contiguous()
        if row_weight is not None:
            row_weight = row_weight.to(device=self.device, dtype=torch.float32).contiguous()
        if out is None:
            out = torch.empty((R, self.cfg.hidden_size), dtype=out_dtype, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_grouped_ffn(self.handle, x_rows.data_ptr(), dtype_code(x_rows.dtype), R,
                                           row_slot.data_ptr(), _ptr(row_weight), out.data_ptr(),
                                           dtype_code(out.dtype), _stream(self.device)))
        return out

    def expert_forward(self, expert_id: int, x: torch.Tensor, *, out_dtype: torch.dtype | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """``RunExpertRequest`` semantics: ``batch`` rows through one expert, fp16/bf16 in and out."""
        x = self._check_x(x)
        od = out_dtype or x.dtype
        if out is None:
            out = torch.empty_like(x, dtype=od)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_expert_forward(self.handle, int(expert_id), x.data_ptr(), dtype_code(x.dtype),
                                              int(x.shape[0]), out.data_ptr(), dtype_code(out.dtype),
                                              _stream(self.device)))
        return out

    def shared_combine(self, x: torch.Tensor, *, extra: torch.Tensor | None = None,
                       residual: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """``out = shared(x) + extra (+ residual)`` cast once (``cst_shared_combine``)."""
        x = self._check_x(x)
        T = x.shape[0]
        if extra is not None:
            if extra.dtype != torch.float32 or extra.shape != x.shape or extra.device != self.device:
                raise RuntimeError("extra must be fp32 [T, hidden] on the context's device")
            extra = extra.contiguous()
        if residual is not None:
            if residual.dtype != x.dtype or residual.shape != x.shape:
                raise RuntimeError("residual must match hidden in shape and dtype")
            residual = residual.contiguous()
        if out is None:
            out = torch.empty((T, self.cfg.hidden_size), dtype=out_dtype or x.dtype, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_shared_combine(self.handle, x.data_ptr(), dtype_code(x.dtype), T, _ptr(extra),
                                              _ptr(residual), out.data_ptr(), dtype_code(out.dtype),
                                              _stream(self.device)))
        return out

    def combine_rows(self, rows: torch.Tensor, tk_row: torch.Tensor, *, extra: torch.Tensor | None = None,
                     residual: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
                     out: torch.Tensor | None = None) -> torch.Tensor:
        """``out[t] = sum_k rows[tk_row[t, k]] (+ extra) (+ residual)`` (``cst_combine_rows``)."""
        T, k1 = tk_row.shape
        tk_row = tk_row.to(device=self.device, dtype=torch.int32).contiguous()
        if rows.dtype != torch.float32 or rows.dim() != 2 or rows.shape[1] != self.cfg.hidden_size:
            raise RuntimeError("rows must be fp32 [*, hidden]")
        if rows.stride(1) != 1:
            rows = rows.contiguous()
        if extra is not None:
            extra = extra.contiguous()
        if residual is not None:
            residual = residual.contiguous()
        if out is None:
            out = torch.empty((T, self.cfg.hidden_size), dtype=out_dtype, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_combine_rows(self.handle, rows.data_ptr(), rows.stride(0), tk_row.data_ptr(), k1, T,
                                            _ptr(extra), _ptr(residual),
                                            dtype_code(residual.dtype) if residual is not None else 0,
                                            out.data_ptr(), dtype_code(out.dtype), _stream(self.device)))
        return out

    def profile(self, enable: bool = True) -> None:
        """Record CUDA events at every stage boundary of the following calls."""
        check(_lib.lib.cst_profile_enable(self.handle, int(bool(enable))))

    def profile_read(self, max_calls: int = 4096) -> list[dict]:
        """Per-call stage durations (ms) recorded since the last read."""
        buf = (ctypes.c_float * (max_calls * _lib.CST_N_STAGES))()
        with torch.cuda.device(self.device):
            n = _lib.lib.cst_profile_read(self.handle, buf, max_calls)
        if n < 0:
            raise _lib.CstError(-n, _lib.last_error())
        vals = list(buf)
        return [dict(zip(_lib.STAGE_NAMES, vals[i * _lib.CST_N_STAGES:(i + 1) * _lib.CST_N_STAGES]))
                for i in range(n)]

    def device_error(self) -> None:
        """Synchronise and raise if a kernel's bounded device-side wait gave up."""
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_device_error(self.handle))
