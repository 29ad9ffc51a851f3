"""Python mirror of the reference's GEMV operator layer over the C ABI.

`Context` owns one chpe_ctx (one CUDA device, one internal stream).  Its
methods keep the reference operators' names and argument meaning:

  gemv_parallel                   src/engine.zig:227-251
  gemv_gate_up_swiglu_parallel    src/engine.zig:285-313
  gemv_batch4_parallel            src/engine.zig:357-391
  gemv_batch8_parallel            src/engine.zig:434-460
  quantize_activation_int8        src/kernels/neon.zig:644-670
  gemv_tile_polymorphic           src/chpe_engine.zig:469-488

They take host numpy arrays and return host arrays, like the reference.  The
device-resident API (`upload_*`, `gemv`, `gemv_gateup_swiglu`) takes torch
CUDA tensors and is asynchronous on the given stream.  Errors raise
ChpeError with the library's message; nothing falls back to the CPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from ._lib import ChpeError


def kernel_launches() -> int:
    """Kernels launched by the library in this process so far (a launch
    recorded into a CUDA graph counts once, at capture)."""
    return int(L.load().chpe_kernel_launches())

def _np_ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return C.c_void_p(a.ctypes.data)


def _dev_ptr(t):
    """Device pointer of a torch tensor (or an int / None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return C.c_void_p(t)
    if isinstance(t, np.ndarray):
        return _np_ptr(t)
    return C.c_void_p(t.data_ptr())


def _stream_ptr(stream):
    if stream is None:
        return None
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(stream.cuda_stream)


class Tensor:
    """A device-resident weight matrix in the strip layout (owned by a Context)."""

    def __init__(self, ctx: "Context", handle: C.c_void_p):
        self.ctx = ctx
        self.handle = handle
        rows, cols, nbytes = L.SZ(), L.SZ(), L.SZ()
        bits = C.c_int()
        ctx._check(ctx.lib.chpe_tensor_info(handle, C.byref(rows), C.byref(cols), C.byref(bits), C.byref(nbytes)))
        self.rows, self.cols, self.bits, self.device_bytes = rows.value, cols.value, bits.value, nbytes.value

    def free(self):
        if self.handle:
            self.ctx._check(self.ctx.lib.chpe_tensor_free(self.ctx.ptr, self.handle))
            self.handle = None

    def unpack(self, n_groups: int | None = None, scales_f32: bool = False, zeros: bool = False):
        """(codes [rows, ceil(cols*bits/8)] uint8, scales, zeros) read back from the
        device layout (chpe_tensor_unpack); scales fp16 [rows, n_groups] (fp32
        [rows] with scales_f32), zeros fp16 when requested, else None."""
        codes = np.zeros((self.rows, (self.cols * self.bits + 7) // 8), np.uint8)
        sc = zz = None
        if scales_f32:
            sc = np.zeros(self.rows, np.float32)
        elif n_groups:
            sc = np.zeros((self.rows, n_groups), np.float16)
        if zeros:
            zz = np.zeros((self.rows, n_groups), np.float16)
        self.ctx._check(self.ctx.lib.chpe_tensor_unpack(self.ctx.ptr, self.handle, _np_ptr(codes),
                                                        None if sc is None else _np_ptr(sc),
                                                        None if zz is None else _np_ptr(zz)))
        return codes, sc, zz

    def __repr__(self):
        return f"Tensor(rows={self.rows}, cols={self.cols}, bits={self.bits}, device_bytes={self.device_bytes})"


class XFrag:
    """Activation fragments shared by several GEMVs over the same input."""

    def __init__(self, ctx: "Context", handle: C.c_void_p, M: int):
        self.ctx, self.handle, self.M = ctx, handle, M

    def free(self):
        if self.handle:
            self.ctx._check(self.ctx.lib.chpe_xfrag_free(self.ctx.ptr, self.handle))
            self.handle = None


class Comm:
    """One-shot NVLink all-reduce of a tensor-parallel group (chpe_comm_*): one
    per rank; `exchange` swaps the IPC handles over any host transport
    (torch.distributed here) and maps every peer's receive area."""

    def __init__(self, ctx: "Context", world: int, rank: int, max_elems: int):
        self.ctx, self.world, self.rank = ctx, world, rank
        h = C.c_void_p()
        ctx._check(ctx.lib.chpe_comm_create(ctx.ptr, world, rank, max_elems, C.byref(h)))
        self.handle = h

    def local_handle(self) -> bytes:
        n = self.ctx.lib.chpe_comm_handle_bytes()
        buf = (C.c_char * n)()
        self.ctx._check(self.ctx.lib.chpe_comm_handle(self.handle, buf))
        return bytes(buf)

    def open_peers(self, handles):
        blob = b"".join(handles)
        buf = (C.c_char * len(blob)).from_buffer_copy(blob)
        self.ctx._check(self.ctx.lib.chpe_comm_open_peers(self.handle, buf))

    def exchange(self, group=None):
        import torch.distributed as dist
        hs = [None] * self.world
        dist.all_gather_object(hs, self.local_handle(), group=group)
        self.open_peers(hs)
        dist.barrier(group=group)

    def allreduce_residual(self, part, hidden, n: int, stream=None):
        """hidden[:n] += sum over ranks of part[:n] (device pointers)."""
        self.ctx._check(self.ctx.lib.chpe_allreduce_residual_dev(self.handle, _dev_ptr(part), _dev_ptr(hidden), n,
                                                                  _stream_ptr(stream)))

    def allreduce_fill(self, part, hidden, xf, gamma, eps: float, stream=None, pushed: bool = False) -> bool:
        """hidden[:M] += sum over ranks of part[:M], then xf = fragments of
        RMSNorm(hidden) * gamma, in one kernel (chpe_allreduce_fill_dev);
        pushed: part came from gemv_push, which sent it already.  False
        (nothing launched) where the fused form does not apply."""
        rc = self.ctx.lib.chpe_allreduce_fill_dev(self.handle, _dev_ptr(part), _dev_ptr(hidden), xf.handle,
                                                  _dev_ptr(gamma), C.c_float(eps), int(pushed), _stream_ptr(stream))
        if rc == L.ENOTSUP:
            return False
        self.ctx._check(rc)
        return True

    def gemv_push(self, w, xf, y, stream=None) -> bool:
        """y = xf . W^T, every output also sent to the peers for the next
        exchange, which must be allreduce_fill(y, ..., pushed=True)
        (chpe_gemv_xfrag_push_dev).  False (nothing launched) for tensors the
        pushing GEMV does not take (outlier columns)."""
        rc = self.ctx.lib.chpe_gemv_xfrag_push_dev(self.ctx.ptr, w.handle, xf.handle, _dev_ptr(y), self.handle,
                                                   _stream_ptr(stream))
        if rc == L.ENOTSUP:
            return False
        self.ctx._check(rc)
        return True

    def argmax_merge(self, idx, maxv, M: int, index_base: int, stream=None):
        """idx[:M] (int32, local to this rank's vocabulary shard) and maxv[:M]
        become the global argmax over the ranks, ties to the smaller index
        (chpe_argmax_merge_dev)."""
        self.ctx._check(self.ctx.lib.chpe_argmax_merge_dev(self.handle, _dev_ptr(idx), _dev_ptr(maxv), M, index_base,
                                                            _stream_ptr(stream)))

    def failed(self) -> bool:
        """True after a bounded wait of this object expired (chpe_comm_failed)."""
        return bool(self.ctx.lib.chpe_comm_failed(self.handle))

    def reset(self, group=None):
        """Resynchronise after a failure: host barrier, chpe_comm_reset on every
        rank, host barrier (no rank exchanges before all ranks have reset)."""
        import torch.distributed as dist
        dist.barrier(group=group)
        self.ctx._check(self.ctx.lib.chpe_comm_reset(self.handle))
        dist.barrier(group=group)

    def close(self):
        if self.handle:
            self.ctx.lib.chpe_comm_destroy(self.handle)
            self.handle = None


class Context:
    def __init__(self, device: int = 0):
        self.lib = L.load()
        self.device = device
        p = C.c_void_p()
        rc = self.lib.chpe_init(device, C.byref(p))
        if rc != 0:
            raise ChpeError(rc, f"chpe_init(device={device}) failed")
        self.ptr = p

    # -- plumbing ------------------------------------------------------------
    def _check(self, rc: int):
        if rc != 0:
            msg = self.lib.chpe_last_error_string(self.ptr)
            raise ChpeError(rc, msg.decode() if msg else "")
        return rc

    def close(self):
        if getattr(self, "ptr", None):
            self.lib.chpe_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self):
        return self._check(self.lib.chpe_sync(self.ptr))

    @staticmethod
    def version() -> str:
        return L.load().chpe_version().decode()

    # -- uploads -------------------------------------------------------------
    def upload_matrix(self, bits: int, scheme: int, codes, scales, zeros=None, bias=None, rows=None, cols=None,
                      group: int = 0, zero: float = 0.0, row_stride: int | None = None) -> Tensor:
        """codes: packed row-major codes (numpy or torch, host or device), rows*row_stride bytes."""
        if rows is None or cols is None:
            raise ValueError("rows and cols are required")
        if row_stride is None:
            row_stride = cols * bits // 8
        f = L.chpe_fmt(bits, scheme, group, zero)
        h = C.c_void_p()
        keep = [codes, scales, zeros, bias]  # noqa: F841  (keep buffers alive during the call)
        # The library reads device inputs on its own stream: whatever torch
        # queued to produce them must have finished first.
        if any(getattr(t, "is_cuda", False) for t in keep):
            import torch
            torch.cuda.current_stream().synchronize()
        self._check(self.lib.chpe_upload_matrix(self.ptr, C.byref(f), _dev_ptr(codes), row_stride, _dev_ptr(scales),
                                                _dev_ptr(zeros), _dev_ptr(bias), rows, cols, C.byref(h)))
        return Tensor(self, h)

    def upload_cells(self, cells, n_cells: int, tile_stride: int = 17408) -> Tensor:
        h = C.c_void_p()
        self._check(self.lib.chpe_upload_cells(self.ptr, _dev_ptr(cells), n_cells, tile_stride, C.byref(h)))
        return Tensor(self, h)

    def quantize_group_dev(self, w, bits: int, group: int, symmetric: bool, stream=None):
        """Device quantizer: returns (codes u8 [rows,cols], scales f16, zeros f16 or None) as torch tensors."""
        import torch
        rows, cols = w.shape
        codes = torch.empty((rows, cols), dtype=torch.uint8, device=w.device)
        scales = torch.empty((rows, cols // group), dtype=torch.float16, device=w.device)
        zeros = None if symmetric else torch.empty((rows, cols // group), dtype=torch.float16, device=w.device)
        self._check(self.lib.chpe_quantize_group_dev(self.ptr, _dev_ptr(w), rows, cols, bits, group, int(symmetric),
                                                     _dev_ptr(codes), _dev_ptr(scales), _dev_ptr(zeros),
                                                     _stream_ptr(stream)))
        return codes, scales, zeros

    # -- device GEMV ------------------------------------------------------------
    def gemv(self, w: Tensor, x, out=None, x_scales=None, accumulate: bool = False, stream=None):
        """y[M, rows] = x[M, cols] . W^T (torch CUDA tensors)."""
        import torch
        x2 = x.reshape(-1, x.shape[-1])
        M = x2.shape[0]
        dt = {torch.float32: L.X_F32, torch.bfloat16: L.X_BF16, torch.float16: L.X_F16, torch.int8: L.X_I8}[x2.dtype]
        if out is None:
            out = torch.empty((M, w.rows), dtype=torch.float32, device=x.device)
        if stream is None:
            stream = torch.cuda.current_stream(x.device)
        self._check(self.lib.chpe_gemv_dev(self.ptr, w.handle, _dev_ptr(x2.contiguous()), dt, _dev_ptr(x_scales), M,
                                           _dev_ptr(out), int(accumulate), _stream_ptr(stream)))
        return out

    def gemv_gateup_swiglu(self, gate: Tensor, up: Tensor, x, out=None, x_scales=None, stream=None):
        import torch
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        M = x2.shape[0]
        dt = {torch.float32: L.X_F32, torch.bfloat16: L.X_BF16, torch.float16: L.X_F16, torch.int8: L.X_I8}[x2.dtype]
        if out is None:
            out = torch.empty((M, gate.rows), dtype=torch.float32, device=x.device)
        if stream is None:
            stream = torch.cuda.current_stream(x.device)
        self._check(self.lib.chpe_gemv_gateup_swiglu_dev(self.ptr, gate.handle, up.handle, _dev_ptr(x2), dt,
                                                         _dev_ptr(x_scales), M, _dev_ptr(out), _stream_ptr(stream)))
        return out

    def quantize_act_i8_dev(self, x, stream=None):
        import torch
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        M, n = x2.shape
        q = torch.empty((M, n), dtype=torch.int8, device=x.device)
        s = torch.empty((M,), dtype=torch.float32, device=x.device)
        if stream is None:
            stream = torch.cuda.current_stream(x.device)
        self._check(self.lib.chpe_quantize_act_i8_dev(self.ptr, _dev_ptr(x2), M, n, _dev_ptr(q), _dev_ptr(s),
                                                      _stream_ptr(stream)))
        return q, s

    # -- shared activation fragments ---------------------------------------------
    def xfrag(self, like: Tensor, M: int, x_dtype: int) -> "XFrag":
        h = C.c_void_p()
        self._check(self.lib.chpe_xfrag_create(self.ptr, like.handle, M, x_dtype, C.byref(h)))
        return XFrag(self, h, M)

    def xfrag_fill(self, xf: "XFrag", x, x_scales=None, stream=None):
        self._check(self.lib.chpe_xfrag_fill_dev(self.ptr, xf.handle, _dev_ptr(x), _dev_ptr(x_scales),
                                                 _stream_ptr(stream)))

    def xfrag_fill_op(self, xf: "XFrag", op: int, x, aux=None, ldx: int = 0, ld_aux: int = 0, eps: float = 0.0,
                      x_dtype: int = L.X_F32, kv_dim: int = 1, head_dim: int = 0, group: int = 1, qkv_dim: int = 1,
                      silu_on_qkv: bool = False, stream=None):
        """Fill fragments from a fused producer (chpe_xfrag_fill_op_dev; L.XOP_*)."""
        s = L.chpe_xsrc(op, _dev_ptr(x), x_dtype, ldx, _dev_ptr(aux), ld_aux, eps, kv_dim, head_dim, group, qkv_dim,
                        int(silu_on_qkv))
        self._check(self.lib.chpe_xfrag_fill_op_dev(self.ptr, xf.handle, C.byref(s), _stream_ptr(stream)))

    def gemv_src(self, tensors, outs, op: int, x, aux=None, M: int = 1, mode: int = 0, accumulate: bool = False,
                 ldx: int = 0, ld_aux: int = 0, eps: float = 0.0, kv_dim: int = 1, head_dim: int = 0, group: int = 1,
                 qkv_dim: int = 1, silu_on_qkv: bool = False, stream=None):
        """GEMV(s) with the activation producer fused in (chpe_gemv_src_dev):
        mode 0: outs[r] (+)= src . tensors[r]^T; mode 1: outs[0] = SwiGLU of
        tensors (gate, up).  src = op(x, aux) as in xfrag_fill_op."""
        s = L.chpe_xsrc(op, _dev_ptr(x), L.X_F32, ldx, _dev_ptr(aux), ld_aux, eps, kv_dim, head_dim, group, qkv_dim,
                        int(silu_on_qkv))
        n = len(tensors)
        hs = (C.c_void_p * n)(*[t.handle for t in tensors])
        ys = (C.c_void_p * n)(*[(_dev_ptr(outs[i]).value if i < len(outs) else None) for i in range(n)])
        self._check(self.lib.chpe_gemv_src_dev(self.ptr, mode, n, hs, C.byref(s), M, ys, int(accumulate),
                                               _stream_ptr(stream)))
        return outs

    def gemv_xfrag(self, w: Tensor, xf: "XFrag", out, accumulate: bool = False, stream=None):
        self._check(self.lib.chpe_gemv_xfrag_dev(self.ptr, w.handle, xf.handle, _dev_ptr(out), int(accumulate),
                                                 _stream_ptr(stream)))
        return out

    def gemm_prefill(self, w: Tensor, x, out=None, accumulate: bool = False, stream=None):
        """y[M, rows] = x[M, cols] . W^T on the tensor cores (chpe_gemm_prefill_dev);
        x is a CUDA tensor (fp32 / bf16 / fp16)."""
        import torch
        M = x.shape[0]
        if out is None:
            out = torch.empty((M, w.rows), dtype=torch.float32, device=x.device)
        dt = {torch.float32: L.X_F32, torch.bfloat16: L.X_BF16, torch.float16: L.X_F16}[x.dtype]
        if stream is None:
            stream = torch.cuda.current_stream(x.device)
        self._check(self.lib.chpe_gemm_prefill_dev(self.ptr, w.handle, _dev_ptr(x.contiguous()), dt, M, _dev_ptr(out),
                                                   out.stride(0), int(accumulate), _stream_ptr(stream)))
        return out

    def gemv_multi_xfrag(self, tensors, xf: "XFrag", outs, stream=None):
        """outs[r] = x . tensors[r]^T for up to 4 tensors of the same cols and
        format, in one launch (chpe_gemv_multi_xfrag_dev)."""
        n = len(tensors)
        hs = (C.c_void_p * n)(*[t.handle for t in tensors])
        ys = (C.c_void_p * n)(*[_dev_ptr(o).value for o in outs])
        self._check(self.lib.chpe_gemv_multi_xfrag_dev(self.ptr, n, hs, xf.handle, ys, _stream_ptr(stream)))
        return outs

    def gemv_gateup_swiglu_xfrag(self, gate: Tensor, up: Tensor, xf: "XFrag", out, stream=None):
        self._check(self.lib.chpe_gemv_gateup_swiglu_xfrag_dev(self.ptr, gate.handle, up.handle, xf.handle,
                                                               _dev_ptr(out), _stream_ptr(stream)))
        return out

    # -- token mixers ----------------------------------------------------------------
    def attn_decode(self, q, k, v, kcache, vcache, pos, M: int, q_heads: int, kv_heads: int, head_dim: int,
                    rope_theta: float, gated: bool, out, ldq: int = 0, ldkv: int = 0, ldo: int = 0, stream=None):
        """GQA decode attention with RoPE over a KV cache (chpe_attn_decode_dev):
        rows 0..M-1 of q / k / v at positions pos .. pos+M-1 (pos a device int32
        tensor); kcache / vcache [max_seq, kv_heads, head_dim] fp32."""
        max_seq = kcache.shape[0]
        self._check(self.lib.chpe_attn_decode_dev(
            self.ptr, _dev_ptr(q), ldq or q.shape[-1], _dev_ptr(k), _dev_ptr(v), ldkv or k.shape[-1],
            _dev_ptr(kcache), _dev_ptr(vcache), _dev_ptr(pos), M, q_heads, kv_heads, head_dim, max_seq,
            C.c_float(rope_theta), int(gated), _dev_ptr(out), ldo or out.shape[-1], _stream_ptr(stream)))
        return out

    def deltanet_step(self, qkv, conv_w, ring, state, decay, pos, M: int, heads: int, key_dim: int, value_dim: int,
                      out, ldqkv: int = 0, ldo: int = 0, stream=None):
        """Gated-DeltaNet conv1d + recurrence over rows 0..M-1 (chpe_deltanet_step_dev)."""
        self._check(self.lib.chpe_deltanet_step_dev(
            self.ptr, _dev_ptr(qkv), ldqkv or qkv.shape[-1], _dev_ptr(conv_w), _dev_ptr(ring), _dev_ptr(state),
            _dev_ptr(decay), _dev_ptr(pos), M, heads, key_dim, value_dim, _dev_ptr(out), ldo or out.shape[-1],
            _stream_ptr(stream)))
        return out

    def pos_advance(self, pos, M: int, stream=None):
        self._check(self.lib.chpe_pos_advance_dev(self.ptr, _dev_ptr(pos), M, _stream_ptr(stream)))

    # -- reference-shaped host operators ----------------------------------------
    def register_i8(self, weights: np.ndarray):
        self._check(self.lib.chpe_register_i8(self.ptr, _np_ptr(weights), weights.shape[0], weights.shape[1]))

    def gemv_parallel(self, weights: np.ndarray, scale_w: float, x_q8: np.ndarray, scale_x: float) -> np.ndarray:
        """src/engine.zig:227-251 gemvParallel (weights [rows, cols] int8)."""
        rows, cols = weights.shape
        out = np.empty(rows, np.float32)
        self._check(self.lib.chpe_gemv_parallel(self.ptr, _np_ptr(weights), scale_w, _np_ptr(x_q8), scale_x, rows,
                                                cols, _np_ptr(out)))
        return out

    def gemv_gate_up_swiglu_parallel(self, gate, scale_gate, up, scale_up, x_q8, scale_x) -> np.ndarray:
        """src/engine.zig:285-313 gemvGateUpSwiGLUParallel."""
        rows, cols = gate.shape
        out = np.empty(rows, np.float32)
        self._check(self.lib.chpe_gemv_gate_up_swiglu_parallel(self.ptr, _np_ptr(gate), scale_gate, _np_ptr(up),
                                                               scale_up, _np_ptr(x_q8), scale_x, rows, cols,
                                                               _np_ptr(out)))
        return out

    def gemv_batch4_parallel(self, weights, scale_w, xs, scales_x):
        """src/engine.zig:357-391 gemvBatch4Parallel; xs is a list of 4 int8 vectors."""
        rows, cols = weights.shape
        outs = [np.empty(rows, np.float32) for _ in range(4)]
        sx = np.ascontiguousarray(scales_x, np.float32)
        self._check(self.lib.chpe_gemv_batch4_parallel(self.ptr, _np_ptr(weights), scale_w, *[_np_ptr(x) for x in xs],
                                                       _np_ptr(sx), rows, cols, *[_np_ptr(o) for o in outs]))
        return outs

    def gemv_batch8_parallel(self, weights, scale_w, xs, scales_x):
        """src/engine.zig:434-460 gemvBatch8Parallel; xs is a list of 8 int8 vectors."""
        rows, cols = weights.shape
        outs = [np.empty(rows, np.float32) for _ in range(8)]
        sx = np.ascontiguousarray(scales_x, np.float32)
        xp = (C.c_void_p * 8)(*[x.ctypes.data for x in xs])
        op = (C.c_void_p * 8)(*[o.ctypes.data for o in outs])
        self._check(self.lib.chpe_gemv_batch8_parallel(self.ptr, _np_ptr(weights), scale_w, C.cast(xp, C.c_void_p),
                                                       _np_ptr(sx), rows, cols, C.cast(op, C.c_void_p)))
        return outs

    def quantize_activation_int8(self, x: np.ndarray):
        """src/kernels/neon.zig:644-670 quantizeActivationInt8 -> (q int8, scale)."""
        x = np.ascontiguousarray(x, np.float32)
        q = np.empty(x.size, np.int8)
        s = C.c_float()
        self._check(self.lib.chpe_quantize_activation_int8(self.ptr, _np_ptr(x), x.size, _np_ptr(q), C.byref(s)))
        return q, np.float32(s.value)

    def gemv_tile_polymorphic(self, cell: np.ndarray, x: np.ndarray, y: np.ndarray, row_base: int = 0,
                              accumulate: bool = False) -> np.ndarray:
        """src/chpe_engine.zig:469-488 gemvTilePolymorphic; writes y[row_base + r]."""
        x = np.ascontiguousarray(x, np.float32)
        self._check(self.lib.chpe_gemv_tile_polymorphic(self.ptr, _np_ptr(cell), _np_ptr(x), x.size, _np_ptr(y),
                                                        row_base, int(accumulate)))
        return y
