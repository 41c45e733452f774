"""The expert node's handling of one InferRequest on a GPU, minus the socket.

``handle_infer_request`` is ``HandleInferRequest`` (``expert_node_v2/worker.cc:83-140``)
with ``BackendWorkspaceCudaV2::RunExpertRequest``
(``backend/cuda/backend_workspace_cuda_v2.cc:19-181``) behind it, over
``cst_serve_infer_request``: one request body in, one response body out.  A body that does
not decode gets no reply (``None``), as the worker drops it.  Otherwise the response echoes
the request's batch_size, hidden_dim and output_dtype with status 1 (no context holds the
expert's layer), 2 (the layer's context does not hold the expert), 4 (an unusable request
or a failed run) or 0 and the expert's output.  Batches of any size up to the context's
row capacity are served in one grouped launch (the reference takes batch 1 only).

``layers[l]`` is the ``ExpertContext`` of layer ``l`` on this GPU (or ``None``); global
expert ids are ``layer * experts_per_layer + local id`` (``server/expert_placement.py:4-24``).
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib
from ._lib import CstInferRequest


def handle_infer_request(layers: Sequence, body: bytes, *, experts_per_layer: int = 256) -> bytes | None:
    body = bytes(body)
    src = (ctypes.c_uint8 * max(len(body), 1)).from_buffer_copy(body or b"\0")
    m = CstInferRequest()
    if _lib.lib.cst_decode_infer_request(ctypes.addressof(src), len(body), ctypes.byref(m)) != _lib.CST_OK:
        return None  # worker.cc:92-97: nothing is sent back
    handles = (ctypes.c_void_p * max(len(layers), 1))(*[None if c is None else c.handle for c in layers])
    layer = m.expert_id // experts_per_layer if m.expert_id >= 0 else -1
    ctx = layers[layer] if 0 <= layer < len(layers) else None
    # a usable request's output has as many bytes as its activation (both 16-bit types)
    cap = _lib.CST_INFER_RESPONSE_FIXED_BYTES + int(m.activation_bytes)
    out = (ctypes.c_uint8 * cap)()
    n = ctypes.c_int64(0)
    args = (handles, len(layers), int(experts_per_layer), ctypes.addressof(src), len(body), ctypes.addressof(out), cap,
            ctypes.byref(n))
    if ctx is None:
        _lib.check(_lib.lib.cst_serve_infer_request(*args, None))  # answered without a device
    else:
        with torch.cuda.device(ctx.device):
            _lib.check(_lib.lib.cst_serve_infer_request(*args, torch.cuda.current_stream(ctx.device).cuda_stream))
    return ctypes.string_at(ctypes.addressof(out), n.value)
