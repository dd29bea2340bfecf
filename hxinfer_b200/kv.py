"""Python front end of the C ABI (include/hx_kv.h) over torch device tensors.

torch supplies device memory and streams only; every computation runs in
libhxkv.so.  Names follow the reference engine: a KV cache per model holding
every layer's K and V, RoPE at a position ("step"), decode attention over
``pos + 1`` positions, prefix snapshots.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib
from ._lib import HX_BF16, HX_FP16, HX_FP32, check, load

_DT = {torch.float16: HX_FP16, torch.float32: HX_FP32}
_SRC_DT = {torch.float16: HX_FP16, torch.float32: HX_FP32, torch.bfloat16: HX_BF16}


def _dt(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return _DT[t.dtype]


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None:
            if not t.is_cuda:
                raise ValueError("tensors must be on a CUDA device")
            if not t.is_contiguous():
                raise ValueError("tensors must be contiguous")


def device_status(clear: bool = True) -> int:
    """Device-side status word (synchronises); raises on a recorded error."""
    rc = load().hx_device_status(1 if clear else 0)
    return check(rc, "device status")


def convert(dst: torch.Tensor, src: torch.Tensor, stream=None):
    """Checkpoint dtype conversion on the device (hx_convert): src (fp16,
    fp32 or bfloat16) into dst (fp16 or fp32), element by element; BF16/FP32
    -> FP16 rounds to nearest even as the reference's loader does, widening is
    exact.  dst may share src's memory when the element sizes match (BF16 ->
    FP16 in place: ``convert(t.view(torch.float16), t)``)."""
    _need_cuda(dst, src)
    if src.dtype not in _SRC_DT:
        raise TypeError(f"unsupported source dtype {src.dtype}")
    if dst.numel() != src.numel():
        raise ValueError(f"{dst.numel()} destination elements for {src.numel()} source elements")
    rc = load().hx_convert(_ptr(dst), _dt(dst), _ptr(src), _SRC_DT[src.dtype], src.numel(),
                           _stream(stream))
    check(rc, "hx_convert")


def decode_kernel_count(n_segments: int, head_dim: int, group: int) -> int:
    """Kernels one hx_decode_attention call launches for n_segments
    (sequence, kv head) pairs, mirroring the library's choice: on the
    head_dim-128 path (group <= 16) the split-K decode kernel, which merges
    its own pieces when 64 <= n_segments <= 16384 and group <= 8, and
    otherwise a combine kernel after it; one generic kernel for other head
    sizes."""
    if head_dim == 128 and group <= 16:
        return 1 if group <= 8 and 64 <= n_segments <= 16384 else 2
    return 1


def prefix_hash(tokens) -> int:
    arr = (C.c_int32 * len(tokens))(*[int(t) for t in tokens])
    return int(load().hx_prefix_hash(arr, len(tokens)))


class RopeTable:
    """Device cos/sin table of the reference RoPE (rope_cpu.cpp:22-25)."""

    def __init__(self, head_dim: int, max_pos: int, theta: float, yarn: dict | None = None):
        cfg = _lib.hx_rope_config(head_dim=head_dim, max_pos=max_pos, theta=theta,
                                  use_yarn=1 if yarn else 0,
                                  yarn_factor=(yarn or {}).get("factor", 1.0),
                                  yarn_beta_fast=(yarn or {}).get("beta_fast", 32.0),
                                  yarn_beta_slow=(yarn or {}).get("beta_slow", 1.0),
                                  yarn_orig_max_pos=(yarn or {}).get("orig_max_pos", 4096))
        h = C.c_void_p()
        check(load().hx_rope_table_create(C.byref(cfg), C.byref(h)), "rope table")
        self.handle = h
        self.head_dim, self.max_pos, self.theta = head_dim, max_pos, theta

    def close(self):
        if self.handle:
            load().hx_rope_table_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def rope_qk(q: torch.Tensor, k: torch.Tensor, num_q_heads: int, num_kv_heads: int,
            head_dim: int, step: int, table: RopeTable, stream=None):
    """In-place RoPE of q [rows, Hq*hd] and k [rows, Hkv*hd] at position `step`."""
    _need_cuda(q, k)
    rows = q.numel() // (num_q_heads * head_dim)
    check(load().hx_rope_qk(_ptr(q), _ptr(k), _dt(q), rows, num_q_heads, num_kv_heads, head_dim,
                            step, table.handle, _stream(stream)), "rope_qk")


class KVCache:
    """Paged head-major fp16 KV cache for every layer of a model (or a shard)."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_seqs: int,
                 max_tokens_per_seq: int, num_blocks: int = 0, *, overlap: bool = False,
                 _handle=None):
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.max_seqs, self.max_tokens_per_seq = max_seqs, max_tokens_per_seq
        if _handle is not None:
            self.handle = _handle
            return
        cfg = _lib.hx_kv_config(num_layers=num_layers, num_kv_heads=num_kv_heads,
                                head_dim=head_dim, max_seqs=max_seqs,
                                max_tokens_per_seq=max_tokens_per_seq, num_blocks=num_blocks,
                                flags=_lib.HX_KV_OVERLAP_LAUNCH if overlap else 0)
        h = C.c_void_p()
        check(load().hx_kv_create(C.byref(cfg), C.byref(h)), "kv create")
        self.handle = h

    @classmethod
    def wrap(cls, k: torch.Tensor, v: torch.Tensor, num_kv_heads: int, head_dim: int,
             capacity: int) -> "KVCache":
        """One-layer, one-sequence cache over caller tensors (head-major inside)."""
        _need_cuda(k, v)
        need = num_kv_heads * capacity * head_dim * 2
        if k.numel() * k.element_size() < need or v.numel() * v.element_size() < need:
            raise ValueError("cache tensors too small")
        h = C.c_void_p()
        check(load().hx_kv_wrap(_ptr(k), _ptr(v), num_kv_heads, head_dim, capacity, C.byref(h)),
              "kv wrap")
        obj = cls(1, num_kv_heads, head_dim, 1, capacity, _handle=h)
        obj._keep = (k, v)
        return obj

    def close(self):
        if getattr(self, "handle", None):
            load().hx_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> dict:
        inf = _lib.hx_kv_info()
        check(load().hx_kv_get_info(self.handle, C.byref(inf)), "kv info")
        return {f: getattr(inf, f) for f, _ in _lib.hx_kv_info._fields_}

    def reserve(self, seq: int, n_tokens: int, stream=None):
        check(load().hx_kv_reserve(self.handle, seq, n_tokens, _stream(stream)), "kv reserve")

    def release(self, seq: int, stream=None):
        check(load().hx_kv_release(self.handle, seq, _stream(stream)), "kv release")

    def write(self, layer: int, seq: int, start: int, k: torch.Tensor, v: torch.Tensor,
              stream=None):
        _need_cuda(k, v)
        n = k.numel() // (self.num_kv_heads * self.head_dim)
        check(load().hx_kv_write(self.handle, layer, seq, start, n, _ptr(k), _ptr(v), _dt(k),
                                 _stream(stream)), "kv write")

    def read(self, layer: int, seq: int, start: int, n: int, stream=None):
        dev = torch.device("cuda", torch.cuda.current_device())
        k = torch.empty((n, self.num_kv_heads, self.head_dim), dtype=torch.float16, device=dev)
        v = torch.empty_like(k)
        check(load().hx_kv_read(self.handle, layer, seq, start, n, _ptr(k), _ptr(v),
                                _stream(stream)), "kv read")
        return k, v

    def fill_normal(self, seed: int, stream=None):
        check(load().hx_kv_fill_normal(self.handle, seed & (2**64 - 1), _stream(stream)),
              "kv fill")

    def rope_append(self, layer: int, k: torch.Tensor, v: torch.Tensor, seq_ids: torch.Tensor,
                    positions: torch.Tensor, *, q: torch.Tensor | None = None,
                    num_q_heads: int = 0, table: RopeTable | None = None, bq=None, bk=None,
                    bv=None, q_out: torch.Tensor | None = None, stream=None):
        _need_cuda(q, k, v, seq_ids, positions, bq, bk, bv, q_out)
        n = seq_ids.numel()
        check(load().hx_rope_append(self.handle, layer, _ptr(q), _ptr(k), _ptr(v), _dt(k), _ptr(bq),
                                    _ptr(bk), _ptr(bv), _ptr(seq_ids), _ptr(positions), n,
                                    num_q_heads, table.handle if table else None, _ptr(q_out),
                                    _dt(q_out) if q_out is not None else HX_FP16,
                                    _stream(stream)), "rope_append")

    def qkv_rope_append(self, layer: int, x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor,
                        wv: torch.Tensor, seq_ids: torch.Tensor, positions: torch.Tensor,
                        num_q_heads: int, *, table: "RopeTable | None" = None,
                        bq=None, bk=None, bv=None, proj_dtype=torch.float16,
                        q_out: torch.Tensor | None = None, stream=None):
        """QKV projection of x [n][hidden] with the reference's fp16 weight
        tensors, fused with bias + RoPE + append (hx_qkv_rope_append); returns
        q_out [n][Hq*head_dim]."""
        _need_cuda(x, wq, wk, wv, seq_ids, positions, q_out, bq, bk, bv)
        n, hidden = x.shape
        if q_out is None:
            q_out = torch.empty((n, num_q_heads * self.head_dim), dtype=torch.float16,
                                device=x.device)
        pdt = HX_FP32 if proj_dtype == torch.float32 else HX_FP16
        check(load().hx_qkv_rope_append(
            self.handle, layer, _ptr(x), _dt(x), hidden, _ptr(wq), _ptr(wk), _ptr(wv), pdt,
            _ptr(bq), _ptr(bk), _ptr(bv), _ptr(seq_ids), _ptr(positions), n, num_q_heads,
            table.handle if table is not None else None, _ptr(q_out), _dt(q_out),
            _stream(stream)), "qkv rope append")
        return q_out

    def workspace_bytes(self, n_seqs: int, num_q_heads: int) -> int:
        return int(load().hx_decode_workspace_bytes(self.handle, n_seqs, num_q_heads))

    def decode(self, layer: int, q: torch.Tensor, seq_ids: torch.Tensor, lengths: torch.Tensor,
               num_q_heads: int, *, scale: float | None = None, out: torch.Tensor | None = None,
               out_dtype=torch.float16, workspace: torch.Tensor | None = None, stream=None):
        _need_cuda(q, seq_ids, lengths, out, workspace)
        n = seq_ids.numel()
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            out = torch.empty((n, num_q_heads * self.head_dim), dtype=out_dtype, device=q.device)
        ws_need = self.workspace_bytes(n, num_q_heads)
        if workspace is None:
            workspace = torch.zeros(max(ws_need, 16), dtype=torch.uint8, device=q.device)
        check(load().hx_decode_attention(self.handle, layer, _ptr(q), _dt(q), _ptr(seq_ids),
                                         _ptr(lengths), n, num_q_heads, scale, _ptr(out), _dt(out),
                                         _ptr(workspace), workspace.numel() * workspace.element_size(),
                                         _stream(stream)), "decode attention")
        return out

    def _append_spec(self, k, v, bq, bk, bv, table):
        return _lib.hx_append_spec(k=_ptr(k), v=_ptr(v), bq=_ptr(bq), bk=_ptr(bk), bv=_ptr(bv),
                                   dtype=_dt(k), table=table.handle if table else None)

    def append_decode(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      seq_ids: torch.Tensor, lengths: torch.Tensor, num_q_heads: int, *,
                      table: "RopeTable | None" = None, bq=None, bk=None, bv=None,
                      scale: float | None = None, out: torch.Tensor | None = None,
                      out_dtype=torch.float16, workspace: torch.Tensor | None = None,
                      stream=None):
        """One decode step in one launch (hx_append_decode_attention): every
        sequence's raw q / k / v rows of the token at position lengths - 1 get
        the bias and RoPE, K / V go into the cache, then attention over
        `lengths` positions.  Equal to rope_append + decode."""
        _need_cuda(q, k, v, seq_ids, lengths, out, workspace, bq, bk, bv)
        n = seq_ids.numel()
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            out = torch.empty((n, num_q_heads * self.head_dim), dtype=out_dtype, device=q.device)
        if workspace is None:
            workspace = torch.zeros(max(self.workspace_bytes(n, num_q_heads), 16),
                                    dtype=torch.uint8, device=q.device)
        spec = self._append_spec(k, v, bq, bk, bv, table)
        check(load().hx_append_decode_attention(
            self.handle, layer, _ptr(q), C.byref(spec), _ptr(seq_ids), _ptr(lengths), n,
            num_q_heads, scale, _ptr(out), _dt(out), _ptr(workspace),
            workspace.numel() * workspace.element_size(), _stream(stream)), "append decode")
        return out

    def decode_gather(self, layer: int, q: torch.Tensor, seq_ids: torch.Tensor,
                      lengths: torch.Tensor, num_q_heads: int, gather: "PeerGather", *,
                      out_offset: int, out_rows: torch.Tensor, out_row_heads: int,
                      out_head0: int, scale: float | None = None,
                      out_dtype=torch.float16, workspace: torch.Tensor | None = None,
                      stream=None):
        """Decode attention of this rank's shard with the outputs stored into
        every rank's gather buffer (hx_decode_attention_gather): q head qh of
        local sequence s lands in row out_rows[s], column block out_head0+qh,
        of the [rows][out_row_heads*head_dim] matrix at byte out_offset.
        Follow it by ``gather.wait(epoch)`` (on every rank) before reading
        the buffer."""
        _need_cuda(q, seq_ids, lengths, out_rows, workspace)
        n = seq_ids.numel()
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if workspace is None:
            workspace = torch.zeros(max(self.workspace_bytes(n, num_q_heads), 16),
                                    dtype=torch.uint8, device=q.device)
        odt = HX_FP32 if out_dtype == torch.float32 else HX_FP16
        check(load().hx_decode_attention_gather(
            self.handle, layer, _ptr(q), _dt(q), _ptr(seq_ids), _ptr(lengths), n, num_q_heads,
            scale, gather.handle, out_offset, _ptr(out_rows), out_row_heads, out_head0, odt,
            _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(stream)),
            "decode attention (gather)")

    def append_decode_gather(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                             seq_ids: torch.Tensor, lengths: torch.Tensor, num_q_heads: int,
                             gather: "PeerGather", *, out_offset: int, out_rows: torch.Tensor,
                             out_row_heads: int, out_head0: int, table: "RopeTable | None" = None,
                             bq=None, bk=None, bv=None, scale: float | None = None,
                             out_dtype=torch.float16, workspace: torch.Tensor | None = None,
                             stream=None):
        """append_decode with the outputs placed as decode_gather places them
        (hx_append_decode_attention_gather)."""
        _need_cuda(q, k, v, seq_ids, lengths, out_rows, workspace, bq, bk, bv)
        n = seq_ids.numel()
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if workspace is None:
            workspace = torch.zeros(max(self.workspace_bytes(n, num_q_heads), 16),
                                    dtype=torch.uint8, device=q.device)
        odt = HX_FP32 if out_dtype == torch.float32 else HX_FP16
        spec = self._append_spec(k, v, bq, bk, bv, table)
        check(load().hx_append_decode_attention_gather(
            self.handle, layer, _ptr(q), C.byref(spec), _ptr(seq_ids), _ptr(lengths), n,
            num_q_heads, scale, gather.handle, out_offset, _ptr(out_rows), out_row_heads,
            out_head0, odt, _ptr(workspace), workspace.numel() * workspace.element_size(),
            _stream(stream)), "append decode (gather)")

    def prefill(self, layer: int, q: torch.Tensor, seq: int, start: int, num_q_heads: int, *,
                scale: float | None = None, out: torch.Tensor | None = None,
                out_dtype=torch.float16, stream=None):
        """Causal attention of q rows [n, Hq*hd] at positions start..start+n-1."""
        _need_cuda(q, out)
        n = q.numel() // (num_q_heads * self.head_dim)
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            out = torch.empty((n, num_q_heads * self.head_dim), dtype=out_dtype, device=q.device)
        check(load().hx_prefill_attention(self.handle, layer, _ptr(q), seq, start, n, num_q_heads,
                                          scale, _ptr(out), _dt(out), _stream(stream)),
              "prefill attention")
        return out

    def snapshot_bytes(self, prefix_len: int) -> int:
        return int(load().hx_snapshot_bytes(self.handle, prefix_len))

    def snapshot(self, seq: int, prefix_len: int, dst: torch.Tensor | None = None, stream=None):
        nbytes = self.snapshot_bytes(prefix_len)
        if dst is None:
            dst = torch.empty(max(nbytes, 16), dtype=torch.uint8,
                              device=torch.device("cuda", torch.cuda.current_device()))
        _need_cuda(dst)
        check(load().hx_kv_snapshot(self.handle, seq, prefix_len, _ptr(dst),
                                    dst.numel() * dst.element_size(), _stream(stream)), "snapshot")
        return dst

    def restore(self, seq: int, prefix_len: int, src: torch.Tensor, stream=None):
        _need_cuda(src)
        check(load().hx_kv_restore(self.handle, seq, prefix_len, _ptr(src),
                                   src.numel() * src.element_size(), _stream(stream)), "restore")


def _handles(caches):
    arr = (C.c_void_p * len(caches))(*[c.handle for c in caches])
    return C.cast(arr, C.POINTER(C.c_void_p)), arr


def snapshot_layers(caches, prefix_len: int, dst: torch.Tensor | None = None, stream=None):
    """hx_kv_snapshot_layers: positions [0, prefix_len) of up to 64 one-layer
    wrapped caches (one per model layer) copied into one buffer, layer i at
    i * snapshot_bytes(prefix_len), in one launch."""
    nbytes = len(caches) * caches[0].snapshot_bytes(prefix_len) if caches else 0
    if dst is None:
        dst = torch.empty(max(nbytes, 16), dtype=torch.uint8,
                          device=torch.device("cuda", torch.cuda.current_device()))
    _need_cuda(dst)
    ptrs, keep = _handles(caches)
    check(load().hx_kv_snapshot_layers(ptrs, len(caches), prefix_len, _ptr(dst),
                                       dst.numel() * dst.element_size(), _stream(stream)),
          "snapshot layers")
    del keep
    return dst


def restore_layers(caches, prefix_len: int, src: torch.Tensor, stream=None):
    """hx_kv_restore_layers: the inverse of snapshot_layers, one launch."""
    _need_cuda(src)
    ptrs, keep = _handles(caches)
    check(load().hx_kv_restore_layers(ptrs, len(caches), prefix_len, _ptr(src),
                                      src.numel() * src.element_size(), _stream(stream)),
          "restore layers")
    del keep


class PeerGather:
    """This rank's gather endpoint (hx_dist_*): a device buffer that every
    rank's decode kernels write into over NVLink peer memory, plus the epoch
    flags the kernels post.  Construct on every rank with the current device
    set; ``exchange`` is a callable that all-gathers one bytes object per
    rank (e.g. built on torch.distributed.all_gather_object) and returns the
    list in rank order."""

    def __init__(self, rank: int, world: int, buffer_bytes: int, exchange):
        lib = load()
        h = C.c_void_p()
        check(lib.hx_dist_create(rank, world, buffer_bytes, C.byref(h)), "dist create")
        self.handle = h
        self.rank, self.world, self.bytes = rank, world, buffer_bytes
        try:
            n = int(lib.hx_dist_handle_bytes())
            mine = (C.c_char * n)()
            check(lib.hx_dist_export(self.handle, mine), "dist export")
            blobs = exchange(bytes(mine))
            if len(blobs) != world or any(len(b) != n for b in blobs):
                raise ValueError("exchange must return one handle per rank")
            allh = (C.c_char * (n * world)).from_buffer_copy(b"".join(blobs))
            check(lib.hx_dist_connect(self.handle, allh), "dist connect")
        except BaseException:
            lib.hx_dist_destroy(self.handle)  # nothing of this rank is in use yet
            self.handle = None
            raise
        self.ptr = int(lib.hx_dist_buffer(self.handle))

    def view(self, dtype=torch.float16, offset: int = 0, shape=None) -> torch.Tensor:
        """A tensor over this rank's buffer (no copy; valid while the endpoint
        lives).  The view must lie inside the buffer."""
        esize = torch.empty((), dtype=dtype).element_size()
        if offset < 0 or offset % esize or offset > self.bytes:
            raise ValueError(f"offset {offset} outside the {self.bytes}-byte buffer or misaligned")
        numel = (self.bytes - offset) // esize
        if shape is not None:
            numel = math.prod(shape)
            if offset + numel * esize > self.bytes:
                raise ValueError(f"a {tuple(shape)} {dtype} view at offset {offset} does not fit "
                                 f"the {self.bytes}-byte buffer")
        storage = torch.cuda.current_device()
        return _tensor_at(self.ptr + offset, numel, dtype, storage, self).view(
            *(shape if shape is not None else (numel,)))

    def wait(self, epoch: int, stream=None):
        """Posts `epoch` to every other rank once the work before it on the
        stream has completed, and holds the stream until every other rank has
        posted it (hx_dist_wait)."""
        check(load().hx_dist_wait(self.handle, epoch & 0xFFFFFFFF, _stream(stream)), "dist wait")

    def close(self):
        """Releases the endpoint.  Synchronise and pass a host barrier first:
        peers may still be writing into this rank's buffer until they have
        waited for the last epoch."""
        if getattr(self, "handle", None):
            check(load().hx_dist_destroy(self.handle), "dist destroy")
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _tensor_at(ptr: int, numel: int, dtype, device: int, owner) -> torch.Tensor:
    """Non-owning tensor over device memory at ptr (keeps `owner` referenced)."""
    class _Holder:
        pass
    holder = _Holder()
    holder.__cuda_array_interface__ = {
        "shape": (numel,), "typestr": {torch.float16: "<f2", torch.float32: "<f4",
                                        torch.uint8: "|u1", torch.int32: "<i4"}[dtype],
        "data": (ptr, False), "version": 3, "strides": None}
    holder.owner = owner
    with torch.cuda.device(device):
        return torch.as_tensor(holder, device=torch.device("cuda", device))
