"""g4attn: host-side mirror of gemma4-webgpu's per-layer attention dispatch over libg4attn.so.

Each method of :class:`Context` replaces one WebGPU dispatch of the reference's attention block
(src/engine.ts:2061-2094) and takes the fields of that shader's ``Params`` uniform as keyword
arguments with the same names.  Tensors are torch CUDA tensors (torch is only the device-memory
and stream plumbing here); the computation runs in the sm_100a kernels of libg4attn.so, called
through its C ABI.  A failing call raises :class:`G4AError` carrying the library's status and
message, as the reference throws when its device is lost (src/engine.ts:2214, 2509).
"""
from __future__ import annotations

import ctypes
from ctypes import c_void_p

from . import _lib
from ._lib import G4AError, call, exported_symbols, load  # noqa: F401

__all__ = ["Context", "G4AError", "load", "exported_symbols", "version", "dist_unique_id", "dist_poll_selftest"]


def version() -> str:
    return load().g4a_version().decode()


def dist_unique_id() -> bytes:
    """A new NCCL unique id (g4a_dist_unique_id): rank 0 makes it and sends it to every rank."""
    buf = (ctypes.c_uint8 * _lib.DIST_ID_BYTES)()
    call("g4a_dist_unique_id", ctypes.cast(buf, c_void_p))
    return bytes(buf)


def dist_poll_selftest(scenario: int, timeout_ms: int) -> tuple[int, int]:
    """Run the communicator deadline logic against the library's fake NCCL (no GPU needed);
    returns (status, aborted)."""
    ab = ctypes.c_int(0)
    st = load().g4a_dist_poll_selftest(int(scenario), int(timeout_ms), ctypes.byref(ab))
    return int(st), int(ab.value)


def _ptr(t) -> c_void_p:
    if t is None:
        return c_void_p(None)
    if isinstance(t, int):
        return c_void_p(t)
    return c_void_p(t.data_ptr())


def _check(t, name, dtype, numel=None, device=None):
    import torch

    if t is None:
        raise ValueError(f"{name} is required")
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{name} has {t.numel()} elements, needs >= {numel}")
    if device is not None and t.device.index != device:
        raise ValueError(f"{name} is on cuda:{t.device.index}, context is on cuda:{device}")


class Context:
    """One libg4attn context: a CUDA device, a stream and the split-KV workspace.

    Mirrors the reference's single GPUDevice/GPUQueue: calls are asynchronous and ordered on
    the context's stream; :meth:`sync` waits with a deadline.  By default the context runs on
    torch's current stream of its device, so torch-allocated buffers and torch CUDA events
    order correctly with the library's kernels.
    """

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        load()
        self.device = device
        self._h = None
        h = c_void_p()
        call("g4a_create", device, ctypes.byref(h))
        self._h = h
        if use_torch_stream:
            import torch

            torch.cuda.set_device(device)
            self.set_stream(torch.cuda.current_stream(device).cuda_stream)

    # ---------------------------------------------------------------- lifetime / plumbing
    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            call("g4a_destroy", self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> c_void_p:
        return self._h

    def set_stream(self, cuda_stream: int | None) -> None:
        """Run on a cudaStream_t handle (0 or None = the legacy default stream)."""
        call("g4a_set_stream", self._h, c_void_p(cuda_stream or None))

    def use_own_stream(self) -> None:
        call("g4a_use_own_stream", self._h)

    def sync(self, timeout_ms: int = 60000) -> None:
        call("g4a_sync", self._h, int(timeout_ms))

    def reserve_workspace(self, max_batch: int, head_dim: int, num_q_heads: int) -> None:
        call("g4a_reserve_workspace", self._h, max_batch, head_dim, num_q_heads)

    # ---------------------------------------------------------------- profiler
    def profile_enable(self, on: bool = True) -> None:
        call("g4a_profile_enable", self._h, 1 if on else 0)

    def profile_reset(self) -> None:
        call("g4a_profile_reset", self._h)

    def profile_read(self, label: str) -> tuple[float, int]:
        """(total device ms, launches) of one kernel label since the last reset."""
        ms = ctypes.c_double()
        n = ctypes.c_uint64()
        call("g4a_profile_read", self._h, label.encode(), ctypes.byref(ms), ctypes.byref(n))
        return ms.value, n.value

    # ---------------------------------------------------------------- producers
    def norm_rope(self, x, weight, rope_freqs=None, *, num_heads, head_dim, eps, position, theta,
                  apply_divisor=0) -> None:
        """fused_per_head_norm_rope.wgsl (src/engine.ts:2078-2084), in place on x f32."""
        import torch

        _check(x, "x", torch.float32, num_heads * head_dim, self.device)
        _check(weight, "weight", torch.float16, head_dim, self.device)
        if apply_divisor:
            _check(rope_freqs, "rope_freqs", torch.float16, head_dim // 2, self.device)
        call("g4a_norm_rope", self._h, _ptr(x), _ptr(weight), _ptr(rope_freqs), num_heads, head_dim,
             float(eps), int(position), float(theta), int(apply_divisor))

    def rms_norm_no_weight(self, x, *, num_heads, head_dim, eps) -> None:
        """per_head_rms_norm_no_weight.wgsl (src/engine.ts:2061-2066), in place."""
        import torch

        _check(x, "x", torch.float32, num_heads * head_dim, self.device)
        call("g4a_rms_norm_no_weight", self._h, _ptr(x), num_heads, head_dim, float(eps))

    def kv_store(self, k, v, k_cache, v_cache, *, num_kv_heads, head_dim, position, max_seq_len,
                 eps=1e-6, fuse_v_norm=1) -> None:
        """kv_cache_store.wgsl (+ fused v_norm) at cache row `position` (= slot)."""
        import torch

        n = num_kv_heads * head_dim
        _check(k, "k", torch.float32, n, self.device)
        _check(v, "v", torch.float32, n, self.device)
        _check(k_cache, "k_cache", torch.float16, max_seq_len * n, self.device)
        _check(v_cache, "v_cache", torch.float16, max_seq_len * n, self.device)
        call("g4a_kv_store", self._h, _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), num_kv_heads, head_dim,
             int(position), max_seq_len, float(eps), int(fuse_v_norm))

    # ---------------------------------------------------------------- attention
    def decode_attn(self, q, k_cache, v_cache, out, *, num_q_heads, num_kv_heads, head_dim, seq_len,
                    scale=1.0, sliding_window=0) -> None:
        """attn_score -> softmax -> attn_output (src/engine.ts:2092-2094); seq_len = kv_len."""
        import torch

        _check(q, "q", torch.float32, num_q_heads * head_dim, self.device)
        _check(k_cache, "k_cache", torch.float16, seq_len * num_kv_heads * head_dim, self.device)
        _check(v_cache, "v_cache", torch.float16, seq_len * num_kv_heads * head_dim, self.device)
        _check(out, "out", torch.float32, num_q_heads * head_dim, self.device)
        call("g4a_decode_attn", self._h, _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), num_q_heads,
             num_kv_heads, head_dim, int(seq_len), float(scale), int(sliding_window))

    def decode_attn_noalloc(self, q, k_cache, v_cache, out, *, num_q_heads, num_kv_heads, head_dim, seq_len,
                            scale=1.0, sliding_window=0) -> None:
        """decode_attn with its split-KV scratch in a fixed static device area: the call
        allocates no memory (no reference counterpart)."""
        import torch

        _check(q, "q", torch.float32, num_q_heads * head_dim, self.device)
        _check(k_cache, "k_cache", torch.float16, seq_len * num_kv_heads * head_dim, self.device)
        _check(v_cache, "v_cache", torch.float16, seq_len * num_kv_heads * head_dim, self.device)
        _check(out, "out", torch.float32, num_q_heads * head_dim, self.device)
        call("g4a_decode_attn_noalloc", self._h, _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), num_q_heads,
             num_kv_heads, head_dim, int(seq_len), float(scale), int(sliding_window))

    def decode_attn_paged(self, q, k_pages, v_pages, page_table, kv_lens, out, *, num_q_heads, num_kv_heads,
                          head_dim, page_size, scale=1.0, sliding_window=0, host_kv_lens=None) -> None:
        """Batched decode over a paged f16 cache (new capability; no reference counterpart)."""
        import numpy as np
        import torch

        batch = kv_lens.numel()
        max_pages = page_table.shape[-1]
        num_pages = k_pages.numel() // (page_size * num_kv_heads * head_dim)
        _check(q, "q", torch.float32, batch * num_q_heads * head_dim, self.device)
        _check(k_pages, "k_pages", torch.float16, None, self.device)
        _check(v_pages, "v_pages", torch.float16, k_pages.numel(), self.device)
        _check(page_table, "page_table", torch.int32, batch * max_pages, self.device)
        _check(kv_lens, "kv_lens", torch.int32, batch, self.device)
        _check(out, "out", torch.float32, batch * num_q_heads * head_dim, self.device)
        hl = c_void_p(None)
        if host_kv_lens is not None:
            arr = np.ascontiguousarray(np.asarray(host_kv_lens, dtype=np.int32))
            if arr.size != batch:
                raise ValueError("host_kv_lens must have one entry per sequence")
            self._host_lens_keepalive = arr
            hl = c_void_p(arr.ctypes.data)
        call("g4a_decode_attn_paged", self._h, _ptr(q), _ptr(k_pages), _ptr(v_pages), _ptr(page_table),
             _ptr(kv_lens), hl, batch, page_size, max_pages, num_pages, num_q_heads, num_kv_heads, head_dim,
             float(scale), int(sliding_window), _ptr(out))

    def decode_attn_partial(self, q, k_cache, v_cache, part, *, num_q_heads, num_kv_heads, head_dim, kv_begin,
                            kv_end, kv_len_total, scale=1.0, sliding_window=0) -> None:
        """Split-KV partial (m | l | o, base-2 max) over positions [kv_begin, kv_end)."""
        import torch

        _check(q, "q", torch.float32, num_q_heads * head_dim, self.device)
        _check(part, "part", torch.float32, num_q_heads * (head_dim + 2), self.device)
        call("g4a_decode_attn_partial", self._h, _ptr(q), _ptr(k_cache), _ptr(v_cache), num_q_heads,
             num_kv_heads, head_dim, int(kv_begin), int(kv_end), int(kv_len_total), float(scale),
             int(sliding_window), _ptr(part))

    def lse_merge(self, parts, n_parts, out, *, num_q_heads, head_dim) -> None:
        import torch

        _check(parts, "parts", torch.float32, n_parts * num_q_heads * (head_dim + 2), self.device)
        _check(out, "out", torch.float32, num_q_heads * head_dim, self.device)
        call("g4a_lse_merge", self._h, _ptr(parts), n_parts, num_q_heads, head_dim, _ptr(out))

    def attn_decode_layer(self, q, k, v, q_norm_w, k_norm_w, rope_freqs, k_cache, v_cache, out, *, num_q_heads,
                          num_kv_heads, head_dim, eps, position, slot, kv_len, max_seq_len, theta,
                          apply_divisor=0, scale=1.0, sliding_window=0, is_producer=1) -> None:
        """The whole attention block of one layer for one token (src/engine.ts:2061-2094)."""
        call("g4a_attn_decode_layer", self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm_w), _ptr(k_norm_w),
             _ptr(rope_freqs), _ptr(k_cache), _ptr(v_cache), _ptr(out), num_q_heads, num_kv_heads, head_dim,
             float(eps), int(position), int(slot), int(kv_len), int(max_seq_len), float(theta),
             int(apply_divisor), float(scale), int(sliding_window), int(is_producer))

    def attn_decode_layer_io(self, qkv_host, qkv_dev, out_dev, out_host, q_norm_w, k_norm_w, rope_freqs, k_cache,
                             v_cache, *, num_q_heads, num_kv_heads, head_dim, eps, position, slot, kv_len,
                             max_seq_len, theta, apply_divisor=0, scale=1.0, sliding_window=0, is_producer=1) -> None:
        """attn_decode_layer with the token's packed q | k | v and the output in (pinned) host
        memory: one call enqueues the copy in, the layer and the copy out."""
        call("g4a_attn_decode_layer_io", self._h, _ptr(qkv_host.data_ptr()), _ptr(qkv_dev), _ptr(out_dev),
             _ptr(out_host.data_ptr()), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope_freqs), _ptr(k_cache),
             _ptr(v_cache), num_q_heads, num_kv_heads, head_dim, float(eps), int(position), int(slot), int(kv_len),
             int(max_seq_len), float(theta), int(apply_divisor), float(scale), int(sliding_window),
             int(is_producer))

    # ---------------------------------------------------------------- memory and IPC
    def alloc(self, nbytes: int) -> int:
        """Device allocation through the library (cudaMalloc); returns the address."""
        p = c_void_p()
        call("g4a_alloc", self._h, int(nbytes), ctypes.byref(p))
        return int(p.value or 0)

    def free(self, dptr: int) -> None:
        call("g4a_free", self._h, c_void_p(dptr))

    def memset(self, dptr: int, value: int, nbytes: int) -> None:
        call("g4a_memset", self._h, c_void_p(dptr), int(value), int(nbytes))

    def ipc_handle(self, dptr: int) -> bytes:
        buf = (ctypes.c_uint8 * 64)()
        call("g4a_ipc_get_handle", self._h, c_void_p(dptr), ctypes.cast(buf, c_void_p))
        return bytes(buf)

    def ipc_open(self, handle: bytes) -> int:
        buf = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
        p = c_void_p()
        call("g4a_ipc_open_handle", self._h, ctypes.cast(buf, c_void_p), ctypes.byref(p))
        return int(p.value or 0)

    def ipc_close(self, dptr: int) -> None:
        call("g4a_ipc_close_handle", self._h, c_void_p(dptr))

    def splitkv_exchange_merge(self, part, rank_buffers: list[int], rank: int, seq: int, out, *, num_q_heads,
                               head_dim) -> None:
        """Push this rank's partial to every rank over peer memory, wait for all, merge (see the
        C header for the protocol)."""
        import torch

        _check(part, "part", torch.float32, num_q_heads * (head_dim + 2), self.device)
        _check(out, "out", torch.float32, num_q_heads * head_dim, self.device)
        arr = (c_void_p * len(rank_buffers))(*[c_void_p(b) for b in rank_buffers])
        call("g4a_splitkv_exchange_merge", self._h, _ptr(part), arr, len(rank_buffers), int(rank), int(seq),
             num_q_heads, head_dim, _ptr(out))

    # ---------------------------------------------------------------- multi-GPU over NCCL
    def dist_init(self, rank: int, nranks: int, unique_id: bytes, timeout_ms: int = 60000) -> None:
        """Create this context's NCCL communicator (g4a_dist_init, non-blocking, deadline)."""
        if len(unique_id) != _lib.DIST_ID_BYTES:
            raise ValueError(f"unique_id must be {_lib.DIST_ID_BYTES} bytes")
        buf = (ctypes.c_uint8 * _lib.DIST_ID_BYTES).from_buffer_copy(unique_id)
        call("g4a_dist_init", self._h, int(rank), int(nranks), ctypes.cast(buf, c_void_p), int(timeout_ms))

    def dist_destroy(self) -> None:
        call("g4a_dist_destroy", self._h)

    def dist_info(self) -> tuple[int, int]:
        r, n = ctypes.c_int(-1), ctypes.c_int(0)
        call("g4a_dist_info", self._h, ctypes.byref(r), ctypes.byref(n))
        return r.value, n.value

    def allgather_partials(self, part, parts_all, floats_per_rank: int, timeout_ms: int = 60000) -> None:
        import torch

        _check(part, "part", torch.float32, floats_per_rank, self.device)
        _check(parts_all, "parts_all", torch.float32, None, self.device)
        call("g4a_allgather_partials", self._h, _ptr(part), _ptr(parts_all), int(floats_per_rank), int(timeout_ms))

    def decode_attn_splitkv(self, q, k_slice, v_slice, parts_all, out, *, num_q_heads, num_kv_heads, head_dim,
                            kv_begin, kv_end, kv_len_total, scale=1.0, sliding_window=0, timeout_ms=60000) -> None:
        """One split-KV step on this rank: partial of its slice, NCCL all-gather, merge (g4a_decode_attn_splitkv)."""
        import torch

        _check(q, "q", torch.float32, num_q_heads * head_dim, self.device)
        _check(k_slice, "k_slice", torch.float16, None, self.device)
        _check(v_slice, "v_slice", torch.float16, None, self.device)
        _check(parts_all, "parts_all", torch.float32, None, self.device)
        _check(out, "out", torch.float32, num_q_heads * head_dim, self.device)
        call("g4a_decode_attn_splitkv", self._h, _ptr(q), _ptr(k_slice), _ptr(v_slice), num_q_heads, num_kv_heads,
             head_dim, int(kv_begin), int(kv_end), int(kv_len_total), float(scale), int(sliding_window),
             _ptr(parts_all), _ptr(out), int(timeout_ms))

    def dist_allgather_host(self, data: bytes, timeout_ms: int = 60000) -> list[bytes]:
        """Synchronous all-gather of equal-sized byte strings over the communicator."""
        n = self.dist_info()[1]
        send = (ctypes.c_uint8 * len(data)).from_buffer_copy(data)
        recv = (ctypes.c_uint8 * (len(data) * max(n, 1)))()
        call("g4a_dist_allgather_host", self._h, ctypes.cast(send, c_void_p), ctypes.cast(recv, c_void_p), len(data),
             int(timeout_ms))
        raw = bytes(recv)
        return [raw[i * len(data):(i + 1) * len(data)] for i in range(n)]

    # ---------------------------------------------------------------- projections
    def matmul(self, weight_format: int, x, weight, scales, out, *, M: int, N: int) -> None:
        """out[m] = sum_k W[m, k] x[k] (g4a_matmul): the Q/K/V and O projections
        (shaders/matmul_quant*.wgsl, matmul_q8*.wgsl, matmul_q4k*.wgsl).  weight_format is
        _lib.WEIGHT_F16 / WEIGHT_Q8 / WEIGHT_Q4K; the packing is g4attn.quant's."""
        import torch

        _check(x, "input", torch.float32, None, self.device)
        _check(out, "out", torch.float32, None, self.device)
        call("g4a_matmul", self._h, int(weight_format), _ptr(x), _ptr(weight), _ptr(scales), _ptr(out), int(M),
             int(N))

    def matmul_group(self, weight_format: int, x, N: int, jobs) -> None:
        """Several matrices over one input in one launch (g4a_matmul_group), as the reference's
        'attn.linearQKV' pass; jobs = [(weight, scales, out, M), ...] (at most 4)."""
        arr = (_lib.MatmulJob * len(jobs))(
            *[_lib.MatmulJob(_ptr(w).value, _ptr(sc).value, _ptr(o).value, int(m)) for (w, sc, o, m) in jobs])
        call("g4a_matmul_group", self._h, int(weight_format), _ptr(x), int(N), arr, len(jobs))

    # ---------------------------------------------------------------- prefill
    def prefill_qkv_prep(self, q, k, v, q_norm_w, k_norm_w, rope_freqs, q16_out, k_cache, v_cache, *, T,
                         start_pos, max_seq_len, num_q_heads, num_kv_heads, head_dim, eps, theta,
                         apply_divisor=0) -> None:
        call("g4a_prefill_qkv_prep", self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm_w), _ptr(k_norm_w),
             _ptr(rope_freqs), _ptr(q16_out), _ptr(k_cache), _ptr(v_cache), int(T), int(start_pos),
             int(max_seq_len), num_q_heads, num_kv_heads, head_dim, float(eps), float(theta), int(apply_divisor))

    def prefill_attn(self, q16, k_cache, v_cache, out, *, T, start_pos, num_q_heads, num_kv_heads, head_dim,
                     scale=1.0, sliding_window=0) -> None:
        call("g4a_prefill_attn", self._h, _ptr(q16), _ptr(k_cache), _ptr(v_cache), _ptr(out), int(T),
             int(start_pos), num_q_heads, num_kv_heads, head_dim, float(scale), int(sliding_window))
