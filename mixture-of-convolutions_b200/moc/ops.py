"""Launch layer: the reference's operator API (moc/ops.py) backed by the C ABI.

Every ``launch_*`` function keeps the reference's name, signature, validation and
output ownership (outputs are allocated here with the torch caching allocator and
passed to the library as raw pointers).  Kernels run on the current torch stream of
the tensors' device.  There is no CPU or Triton fallback.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

VARLEN_BLOCK_T = 64
_CHUNK_CACHE_SIZE = 4
# entries: (cu_seqlens, version, chunk_size, cu_seqlens_cpu, cpu_version, chunk_indices)
_chunk_index_cache: list[tuple] = []


def _tensor_version(t: torch.Tensor | None) -> int | None:
    return None if t is None else t._version


def clear_chunk_index_cache() -> None:
    """Drop every cached chunk table (reference: moc/ops.py:43-44)."""
    _chunk_index_cache.clear()


def _chunk_count_table(cu_host: torch.Tensor, chunk_size: int) -> torch.Tensor:
    lengths = cu_host[1:].to(torch.int64) - cu_host[:-1].to(torch.int64)
    counts = torch.div(lengths + chunk_size - 1, chunk_size, rounding_mode="floor")
    if bool((counts < 0).any()):
        raise RuntimeError("repeats can not be negative")
    return counts


def prepare_chunk_indices(
    cu_seqlens: torch.Tensor,
    chunk_size: int = VARLEN_BLOCK_T,
    cu_seqlens_cpu: torch.Tensor | None = None,
) -> torch.Tensor:
    """int32 [n_chunks, 2] table of (seq_id, chunk_in_seq) for chunk_size-token chunks.

    Same contract and 4-entry LRU as the reference (moc/ops.py:47-104), keyed by tensor
    identity and version.  The table itself is written on the device by
    ``moc_prepare_chunk_indices``; only the chunk count comes from the host, read from
    ``cu_seqlens_cpu`` when given (no device sync) or from ``cu_seqlens`` otherwise.
    """
    if not isinstance(chunk_size, int) or chunk_size <= 0:
        raise ValueError("chunk_size must be a positive Python int")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be rank-1 with at least two entries")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError("cu_seqlens must have dtype torch.int32 or torch.int64")
    if cu_seqlens_cpu is not None:
        if cu_seqlens_cpu.device.type != "cpu":
            raise ValueError("cu_seqlens_cpu must be a CPU tensor")
        if cu_seqlens_cpu.ndim != 1 or cu_seqlens_cpu.numel() != cu_seqlens.numel():
            raise ValueError("cu_seqlens_cpu must match cu_seqlens shape")
        if cu_seqlens_cpu.dtype not in (torch.int32, torch.int64):
            raise TypeError("cu_seqlens_cpu must have dtype torch.int32 or torch.int64")

    key_version = _tensor_version(cu_seqlens)
    key_cpu_version = _tensor_version(cu_seqlens_cpu)
    for pos, (c_cu, c_ver, c_size, c_cpu, c_cpu_ver, c_table) in enumerate(_chunk_index_cache):
        if (
            c_cu is cu_seqlens
            and c_ver == key_version
            and c_size == chunk_size
            and c_cpu is cu_seqlens_cpu
            and c_cpu_ver == key_cpu_version
        ):
            if pos:
                _chunk_index_cache.insert(0, _chunk_index_cache.pop(pos))
            return c_table

    host = cu_seqlens_cpu if cu_seqlens_cpu is not None else cu_seqlens.detach().cpu()
    counts = _chunk_count_table(host, chunk_size)
    n_chunks = int(counts.sum())
    if cu_seqlens.device.type != "cuda":
        # Host bookkeeping for host offsets: the same table, built with tensor ops.
        seq_ids = torch.repeat_interleave(torch.arange(counts.numel(), dtype=torch.int64), counts)
        first = torch.cumsum(counts, 0) - counts
        within = torch.arange(n_chunks, dtype=torch.int64) - first[seq_ids]
        table = torch.stack((seq_ids, within), dim=1).to(torch.int32).contiguous()
    else:
        table = torch.empty((n_chunks, 2), dtype=torch.int32, device=cu_seqlens.device)
    if n_chunks > 0 and cu_seqlens.device.type == "cuda":
        cu = cu_seqlens.contiguous()
        with torch.cuda.device(cu.device):
            rc = _lib.load().moc_prepare_chunk_indices(
                _lib.ptr(cu), _lib.index_code(cu), cu.numel() - 1, chunk_size,
                _lib.ptr(table), n_chunks, _lib.stream_of(cu.device),
            )
        _lib.check(rc, "moc_prepare_chunk_indices")

    _chunk_index_cache.insert(
        0, (cu_seqlens, key_version, chunk_size, cu_seqlens_cpu, key_cpu_version, table)
    )
    del _chunk_index_cache[_CHUNK_CACHE_SIZE:]
    return table


def chunk_indices_upper_bound(cu_seqlens: torch.Tensor, n_tokens: int, chunk_size: int = VARLEN_BLOCK_T) -> torch.Tensor:
    """int32 [n_tokens // chunk_size + n_seqs, 2] chunk table built on the device without
    reading cu_seqlens on the host: no stream synchronisation, so a varlen forward and
    backward can be captured in a CUDA graph.

    The sum of ceil(len_i / chunk_size) over the n_seqs sequences of n_tokens tokens is at
    most n_tokens // chunk_size + n_seqs, so a table of that many rows holds every chunk of
    the reference's table (moc/ops.py:82-97), in the same order; the rows after the last
    chunk are (-1, -1), which the kernels skip.  Outside stream capture the table is kept
    in the same 4-entry LRU as ``prepare_chunk_indices``; during capture it is always built
    in the graph's own memory, so the graph never depends on a table the LRU may drop.
    """
    n_seqs = cu_seqlens.numel() - 1
    rows = int(n_tokens) // chunk_size + n_seqs
    capturing = torch.cuda.is_current_stream_capturing()
    key = ("bound", int(n_tokens))
    version = _tensor_version(cu_seqlens)
    if not capturing:
        for pos, (c_cu, c_ver, c_size, c_cpu, c_cpu_ver, c_table) in enumerate(_chunk_index_cache):
            if (c_cu is cu_seqlens and c_ver == version and c_size == chunk_size and isinstance(c_cpu, tuple)
                    and c_cpu == key):
                if pos:
                    _chunk_index_cache.insert(0, _chunk_index_cache.pop(pos))
                return c_table
    table = torch.empty((rows, 2), dtype=torch.int32, device=cu_seqlens.device)
    if rows > 0:
        cu = cu_seqlens.contiguous()
        with torch.cuda.device(cu.device):
            rc = _lib.load().moc_prepare_chunk_indices(
                _lib.ptr(cu), _lib.index_code(cu), n_seqs, chunk_size, _lib.ptr(table), rows,
                _lib.stream_of(cu.device),
            )
        _lib.check(rc, "moc_prepare_chunk_indices")
    if not capturing:
        _chunk_index_cache.insert(0, (cu_seqlens, version, chunk_size, key, None, table))
        del _chunk_index_cache[_CHUNK_CACHE_SIZE:]
    return table


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous and 16-byte aligned (the vectorised kernels stage rows in 16 B chunks)."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _check_chunk_indices(chunk_indices: torch.Tensor, cu_seqlens: torch.Tensor) -> None:
    if not chunk_indices.is_cuda or chunk_indices.device != cu_seqlens.device:
        raise ValueError("chunk_indices must be a CUDA tensor on the same device as cu_seqlens")
    if chunk_indices.ndim != 2 or chunk_indices.shape[1] != 2:
        raise ValueError("chunk_indices must have shape [num_chunks, 2]")
    if chunk_indices.dtype not in (torch.int32, torch.int64):
        raise TypeError("chunk_indices must have dtype torch.int32 or torch.int64")
    if not chunk_indices.is_contiguous():
        raise ValueError("chunk_indices must be contiguous")


def _problem(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    activation_flag: int,
    cu_seqlens: torch.Tensor | None,
    cu_seqlens_cpu: torch.Tensor | None,
    chunk_indices: torch.Tensor | None,
    block_t: int,
    halo: torch.Tensor | None = None,
) -> tuple[_lib.MocProblem, tuple]:
    """Fill a moc_problem; returns it with the tensors that must outlive the call."""
    K, S, D = basis.shape
    p = _lib.MocProblem()
    p.dim = D
    p.n_bases = K
    p.kernel_size = S
    p.x_dtype = _lib.dtype_code(x)
    p.alpha_dtype = _lib.dtype_code(alpha)
    p.basis_dtype = _lib.dtype_code(basis)
    p.activation = int(activation_flag)
    keep: tuple = ()
    if cu_seqlens is not None:
        if chunk_indices is None:
            if cu_seqlens_cpu is not None:
                chunk_indices = prepare_chunk_indices(cu_seqlens, block_t, cu_seqlens_cpu)
            else:  # no host copy of the offsets: a bound-sized table, no device sync
                chunk_indices = chunk_indices_upper_bound(cu_seqlens, x.shape[0], block_t)
        _check_chunk_indices(chunk_indices, cu_seqlens)
        cu = cu_seqlens.contiguous()
        p.batch = 0
        p.seq_len = 0
        p.n_tokens = x.shape[0]
        p.cu_seqlens = _lib.ptr(cu)
        p.cu_seqlens_dtype = _lib.index_code(cu)
        p.n_seqs = cu.numel() - 1
        p.chunk_indices = _lib.ptr(chunk_indices)
        p.chunk_indices_dtype = _lib.index_code(chunk_indices)
        p.n_chunks = chunk_indices.shape[0]
        p.chunk_size = int(block_t)
        keep = (cu, chunk_indices)
    else:
        B, T, _ = x.shape
        p.batch = B
        p.seq_len = T
        p.n_tokens = B * T
        if halo is not None:
            if halo.shape != (B, D, S) or halo.dtype != x.dtype or halo.device != x.device:
                raise ValueError(f"halo must be a [{B}, {D}, {S}] {x.dtype} tensor on x's device")
            p.halo = _lib.ptr(halo)
            for i, st in enumerate(halo.stride()):
                p.halo_strides[i] = st
            keep = (halo,)
    return p, keep


def launch_forward(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    *,
    activation_flag: int,
    cu_seqlens: torch.Tensor | None = None,
    cu_seqlens_cpu: torch.Tensor | None = None,
    chunk_indices: torch.Tensor | None = None,
    block_t: int = VARLEN_BLOCK_T,
    halo: torch.Tensor | None = None,
) -> torch.Tensor:
    """y = [silu](conv(x, alpha, basis)) in x.dtype (reference: moc/ops.py:129-194).

    ``halo`` (an extension, fixed length only): the conv cache [B, D, S] of the tokens
    before each sequence, read by the first S-1 positions' taps instead of zeros."""
    x, alpha, basis = _aligned(x), _aligned(alpha), _aligned(basis)
    out = torch.empty_like(x)
    p, keep = _problem(x, alpha, basis, activation_flag, cu_seqlens, cu_seqlens_cpu, chunk_indices, block_t, halo)
    with torch.cuda.device(x.device):
        rc = _lib.load().moc_forward(
            ctypes.byref(p), _lib.ptr(x), _lib.ptr(alpha), _lib.ptr(basis), _lib.ptr(out),
            _lib.stream_of(x.device),
        )
    _lib.check(rc, "moc_forward")
    del keep
    return out


def launch_preact(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    *,
    cu_seqlens: torch.Tensor | None = None,
    cu_seqlens_cpu: torch.Tensor | None = None,
    chunk_indices: torch.Tensor | None = None,
    block_t: int = VARLEN_BLOCK_T,
) -> torch.Tensor:
    """Forward without the activation (reference: moc/ops.py:197-213)."""
    return launch_forward(
        x, alpha, basis, activation_flag=0, cu_seqlens=cu_seqlens,
        cu_seqlens_cpu=cu_seqlens_cpu, chunk_indices=chunk_indices, block_t=block_t,
    )


def launch_backward(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    moc_dy: torch.Tensor,
    preact: torch.Tensor,
    *,
    activation_flag: int,
    need_x: bool,
    cu_seqlens: torch.Tensor | None = None,
    cu_seqlens_cpu: torch.Tensor | None = None,
    chunk_indices: torch.Tensor | None = None,
    block_t: int = VARLEN_BLOCK_T,
    halo: torch.Tensor | None = None,
) -> tuple[torch.Tensor | None, torch.Tensor, torch.Tensor]:
    """(dx | None, dalpha, dbasis) (reference: moc/ops.py:216-338).

    With ``activation_flag`` set the kernels recompute the pre-activation on chip in
    fp32, so ``preact`` is accepted for signature compatibility but not read.  dbasis
    is reduced deterministically (per-CTA fp32 partials summed in a fixed order).
    ``halo`` as in launch_forward (the cache gets no gradient).
    """
    del preact
    x, alpha, basis, moc_dy = _aligned(x), _aligned(alpha), _aligned(basis), _aligned(moc_dy)
    p, keep = _problem(x, alpha, basis, activation_flag, cu_seqlens, cu_seqlens_cpu, chunk_indices, block_t, halo)
    lib = _lib.load()
    dx = torch.empty_like(x) if need_x else None
    dalpha = torch.empty_like(alpha)
    dbasis = torch.empty_like(basis)
    ws_bytes = lib.moc_backward_workspace_bytes(ctypes.byref(p))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib.moc_backward(
            ctypes.byref(p), _lib.ptr(x), _lib.ptr(alpha), _lib.ptr(basis), _lib.ptr(moc_dy),
            _lib.ptr(dx), _lib.ptr(dalpha), _lib.ptr(dbasis), _lib.ptr(ws), ws_bytes,
            _lib.stream_of(x.device),
        )
    _lib.check(rc, "moc_backward")
    del keep
    return dx, dalpha, dbasis


def launch_update(
    x: torch.Tensor,
    alpha: torch.Tensor,
    basis: torch.Tensor,
    cache: torch.Tensor,
    *,
    activation_flag: int,
) -> torch.Tensor:
    """Decode step: y [B,D]; shifts ``cache`` [B,D,S] in place and appends x
    (reference: moc/ops.py:341-362, kernel moc/kernels.py:442-550)."""
    x = x.contiguous()
    alpha = alpha.contiguous()
    basis = basis.contiguous()
    B, D = x.shape
    K, S, _ = basis.shape
    out = torch.empty_like(x)
    strides = (ctypes.c_int64 * 3)(*cache.stride())
    with torch.cuda.device(x.device):
        rc = _lib.load().moc_step(
            B, D, K, S, _lib.dtype_code(x), _lib.dtype_code(alpha), _lib.dtype_code(basis),
            int(activation_flag), _lib.ptr(x), _lib.ptr(alpha), _lib.ptr(basis), _lib.ptr(cache),
            strides, _lib.ptr(out), _lib.stream_of(x.device),
        )
    _lib.check(rc, "moc_step")
    return out


# ----------------------------------------------------------------------------- router

ROUTER_ACTIVATIONS = {"softmax": 0, "exp": 1}


def launch_router_forward(z: torch.Tensor, weight: torch.Tensor, router_activation: str) -> torch.Tensor:
    """alpha = softmax(z @ weight^T) or exp(z @ weight^T), fp32 logits, z.dtype output.

    Replaces ``F.linear`` + ``torch.softmax``/``torch.exp`` of MoC.forward
    (reference: moc/api.py:383-388).
    """
    z2 = z.reshape(-1, z.shape[-1]).contiguous()
    weight = weight.contiguous()
    K, Dz = weight.shape
    alpha = torch.empty((z2.shape[0], K), dtype=z.dtype, device=z.device)
    with torch.cuda.device(z.device):
        rc = _lib.load().moc_router_forward(
            z2.shape[0], Dz, K, _lib.dtype_code(z2), ROUTER_ACTIVATIONS[router_activation],
            _lib.ptr(z2), _lib.ptr(weight), _lib.ptr(alpha), _lib.stream_of(z.device),
        )
    _lib.check(rc, "moc_router_forward")
    return alpha.reshape(*z.shape[:-1], K)


def launch_router_backward(
    z: torch.Tensor,
    weight: torch.Tensor,
    alpha: torch.Tensor,
    dalpha: torch.Tensor,
    router_activation: str,
    *,
    need_z: bool = True,
    need_weight: bool = True,
) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """(dz, dweight) from dalpha through the softmax/exp Jacobian and the router GEMM."""
    z2 = z.reshape(-1, z.shape[-1]).contiguous()
    weight = weight.contiguous()
    K, Dz = weight.shape
    a2 = alpha.reshape(-1, K).contiguous()
    da2 = dalpha.reshape(-1, K).contiguous()
    N = z2.shape[0]
    lib = _lib.load()
    dz = torch.empty_like(z2) if need_z else None
    dw = torch.empty_like(weight) if need_weight else None
    code = _lib.dtype_code(z2)
    ws_bytes = lib.moc_router_backward_workspace_bytes(N, Dz, K, code)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=z.device)
    with torch.cuda.device(z.device):
        rc = lib.moc_router_backward(
            N, Dz, K, code, ROUTER_ACTIVATIONS[router_activation], _lib.ptr(z2), _lib.ptr(weight),
            _lib.ptr(a2), _lib.ptr(da2), _lib.dtype_code(da2), _lib.ptr(dz), _lib.ptr(dw),
            _lib.ptr(ws), ws_bytes, _lib.stream_of(z.device),
        )
    _lib.check(rc, "moc_router_backward")
    return (None if dz is None else dz.reshape(z.shape)), dw
