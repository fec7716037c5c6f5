"""tp -- tensor-parallel drivers of the quantized-linear GEMMs, one process per GPU.

Mirrors the two sharded linears of kernel-craft's tensor_parallel.cu for the
quantized GEMMs, with the processes of one node as ranks (the reference runs
every rank inside one process, tensor_parallel.cu:209-243 and
tensor_parallel_nccl.cu:105-135):

* column parallel (``launch_col_parallel_linear`` + ``launch_allgather_nccl``):
  rank r owns weight rows [r*N/R, (r+1)*N/R) of a W4A16 matrix; the activations
  are replicated.  ``ColParallelW4A16`` runs the fused kernel
  ``kc_gemm_w4a16_allgather``: its epilogue writes every output tile straight
  into all ranks' [M, N] buffers over NVLink, so the all-gather costs no
  separate pass and the result lands in [M, N] order (the reference gathers
  rank-major blocks).
* row parallel (``launch_row_parallel_linear`` + ``launch_ring_allreduce_nccl``):
  rank r owns columns [r*K/R, (r+1)*K/R) of the FP8 codes of both operands (the
  per-token and per-channel scales come from the full rows, so each partial
  already carries the scale epilogue, which is linear); ``RowParallelFP8``
  runs ``kc_gemm_fp8`` on the shard and sums the bf16 partials with
  ``kc_allreduce_bf16_peer`` over NVLink peer memory (each rank reduces one
  slice from all partials and writes it to every rank); ``row_parallel_fp8``
  is the same linear with an NCCL all-reduce instead.

* the MLP block (the reference's col-parallel -> GELU -> row-parallel chain,
  examples/python/transformer/tensor_parallel.py:150-172): ``MLPBlockW4A16``
  runs the up projection on its rows of W1 with the GELU in the GEMM epilogue
  (``kc_gemm_w4a16_act``), the down projection on the same columns of W2 into
  an fp32 partial, and one all-reduce; no communication between the two GEMMs.

The process group must be NCCL for the GPU collectives; every rank calls the
same functions in the same order.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Tuple

import torch
import torch.distributed as dist

import kc_lib
from kc_lib import check, lib


def shard_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """[begin, end) of rank's equal share of `total`; `total` must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if total % world:
        raise ValueError(f"{total} does not split evenly over {world} ranks")
    share = total // world
    return rank * share, (rank + 1) * share


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def barrier_on_stream(group=None) -> None:
    """Stream-ordered barrier: a one-element all-reduce on the current stream,
    so work queued after it on any rank starts only when every rank's
    preceding work has finished."""
    flag = torch.zeros(1, dtype=torch.float32, device="cuda")
    dist.all_reduce(flag, group=group)


def check_operand(t: torch.Tensor, name: str, shape, dtypes, cuda: bool = True) -> None:
    """Raise ValueError unless t is a contiguous tensor of the given shape and
    one of the given dtypes (on a CUDA device when cuda): the kernels receive
    raw pointers and sizes, so a mismatched shard would be read out of
    bounds instead of failing."""
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name}: expected a torch.Tensor, got {type(t).__name__}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
    if t.dtype not in dtypes:
        raise ValueError(f"{name}: dtype {t.dtype}, expected one of {[str(d) for d in dtypes]}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    if cuda and not t.is_cuda:
        raise ValueError(f"{name}: must be on a CUDA device")


_BF16 = (torch.bfloat16, torch.int16)         # bf16 bits may arrive as int16
_F16 = (torch.float16, torch.int16)
_U8 = (torch.uint8,)
_I8 = (torch.int8, torch.uint8)


def check_col_parallel_w4a16(M, K, n_shard, gs, x, packed_shard, scales_shard, cuda=True):
    check_operand(x, "x", (M, K), _BF16, cuda)
    check_operand(packed_shard, "packed_shard", (n_shard, K // 2), _U8, cuda)
    check_operand(scales_shard, "scales_shard", (n_shard, K // gs), _F16, cuda)


def check_row_parallel_fp8(M, N, a_codes_shard, sa, w_codes_shard, sw, cuda=True):
    if a_codes_shard.dim() != 2:
        raise ValueError("a_codes_shard must be 2-D")
    kr = a_codes_shard.shape[1]
    check_operand(a_codes_shard, "a_codes_shard", (M, kr), _I8, cuda)
    check_operand(w_codes_shard, "w_codes_shard", (N, kr), _I8, cuda)
    check_operand(sa, "sa", (M,), (torch.float32,), cuda)
    check_operand(sw, "sw", (N,), (torch.float32,), cuda)


def check_mlp_block_w4a16(M, H, i_shard, gs, x, w1_packed, w1_scales, w2_packed, w2_scales, cuda=True):
    check_operand(x, "x", (M, H), _BF16, cuda)
    check_operand(w1_packed, "w1_packed", (i_shard, H // 2), _U8, cuda)
    check_operand(w1_scales, "w1_scales", (i_shard, H // gs), _F16, cuda)
    check_operand(w2_packed, "w2_packed", (H, i_shard // 2), _U8, cuda)
    check_operand(w2_scales, "w2_scales", (H, i_shard // gs), _F16, cuda)


def barrier_timeout_s() -> float:
    """Bound of every peer-barrier wait, in seconds: $KC_PEER_BARRIER_TIMEOUT_S,
    else 30 s -- long enough for a rank that stalls on the host between
    steps (a checkpoint load, a first-call module load, a garbage
    collection) to arrive late without the barrier giving up."""
    return float(os.environ.get("KC_PEER_BARRIER_TIMEOUT_S", "30"))


class PeerBarrier:
    """Stream-ordered barrier over peer memory (kc_peer_barrier): a one-warp
    kernel per rank exchanges an increasing epoch through flag arrays shared
    with CUDA IPC; cheaper than a one-element NCCL collective.

    Each wait is bounded (``timeout_s``, default ``barrier_timeout_s()``).  A
    wait that gives up leaves the results around it undefined; the kernel
    then writes KC_ERR_TIMEOUT into a pinned host slot, and the next call of
    this barrier -- or ``check()`` at a sync point -- raises ``KcError``
    (the peer all-reduce writes NaN meanwhile)."""

    def __init__(self, group=None, timeout_s: float | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.timeout_ns = int((barrier_timeout_s() if timeout_s is None else timeout_s) * 1e9)
        self.bufs = PeerBuffers(kc_lib.KC_MAX_RANKS * 4, group)
        self.bufs.local((kc_lib.KC_MAX_RANKS,), torch.int32).zero_()
        # written by the device when a wait gives up; read here without a sync
        self.status = torch.zeros(1, dtype=torch.int32).pin_memory()
        torch.cuda.synchronize()
        dist.barrier(group=group)          # every flag array is zero before first use
        self._flags = (ctypes.c_void_p * self.world)(*self.bufs.ptrs)
        self.epoch = 0

    def check(self) -> None:
        """Raise KcError if any earlier wait of this barrier gave up (only
        waits that have already run on the device are seen: synchronize
        first for a complete answer)."""
        st = int(self.status[0])
        if st != kc_lib.KC_OK:
            raise kc_lib.KcError(st, f"a peer barrier of rank {self.rank} gave up after "
                                     f"{self.timeout_ns / 1e9:.1f} s: the results of the calls "
                                     "since are undefined (kc_get_device_status() clears the "
                                     "device status)")

    def __call__(self) -> None:
        self.check()
        self.epoch += 1
        check(lib().kc_peer_barrier(self._flags, self.world, self.rank, self.epoch,
                                    self.timeout_ns, ctypes.c_void_p(self.status.data_ptr()),
                                    _stream()))

    def close(self) -> None:
        torch.cuda.synchronize()
        self.bufs.close()


class PeerBuffers:
    """One device buffer per rank, every rank mapping every other rank's buffer
    (CUDA IPC through the kc_ipc_* entry points; handles travel over the
    process group).  ``ptrs[r]`` is rank r's buffer as seen from this process;
    ``local`` wraps this rank's own buffer as a torch tensor view."""

    def __init__(self, nbytes: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > kc_lib.KC_MAX_RANKS:
            raise ValueError(f"at most {kc_lib.KC_MAX_RANKS} ranks")
        l = lib()
        own = ctypes.c_void_p()
        check(l.kc_ipc_alloc(ctypes.byref(own), nbytes))
        self._own = own
        hb = l.kc_ipc_handle_bytes()
        handle = (ctypes.c_char * hb)()
        check(l.kc_ipc_get_handle(own, handle))
        handles: List[bytes] = [b""] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs: List[int] = []
        self._opened: List[ctypes.c_void_p] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(own.value)
                continue
            p = ctypes.c_void_p()
            check(l.kc_ipc_open(ctypes.create_string_buffer(h, hb), ctypes.byref(p)))
            self._opened.append(p)
            self.ptrs.append(p.value)
        self.nbytes = nbytes

    def local(self, shape, dtype) -> torch.Tensor:
        """This rank's buffer as a CUDA tensor (no copy; valid until close())."""
        n = 1
        for d in shape:
            n *= d
        if n * torch.empty((), dtype=dtype).element_size() > self.nbytes:
            raise ValueError("view larger than the buffer")
        return _from_blob(self._own.value, shape, dtype, torch.cuda.current_device())

    def close(self) -> None:
        """Unmaps the peers' buffers, waits for every rank, frees our own."""
        l = lib()
        for p in self._opened:
            l.kc_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        if self._own:
            l.kc_ipc_free(self._own)
            self._own = ctypes.c_void_p()


class SymmetricBuffer:
    """A device buffer allocated on every rank and bound to one NVLink
    multicast object (torch's symmetric memory does the allocation, the
    handle exchange and the binding): ``local`` is this rank's copy,
    ``multicast_ptr`` the address through which multimem instructions reach
    every rank's copy at once.  Raises RuntimeError where the platform offers
    no multicast (no NVSwitch, or a driver without it)."""

    def __init__(self, shape, dtype, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group
        grp = group if group is not None else dist.group.WORLD
        n = 1
        for d in shape:
            n *= d
        flat = symm_mem.empty(n, dtype=dtype, device=torch.device("cuda", torch.cuda.current_device()))
        self.handle = symm_mem.rendezvous(flat, grp)
        self.local = flat.view(tuple(shape))
        self.multicast_ptr = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        if not self.multicast_ptr:
            raise RuntimeError("no NVLink multicast on this platform (symmetric memory has no "
                               "multicast address)")
        if self.multicast_ptr % 16:
            raise RuntimeError("multicast address not 16-byte aligned")

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.handle = None
        self.local = None


def _from_blob(ptr: int, shape, dtype, device: int) -> torch.Tensor:
    """A tensor viewing device memory owned elsewhere (lifetime managed by the
    caller), through the __cuda_array_interface__ protocol."""
    typestr, view = {torch.bfloat16: ("<i2", torch.bfloat16), torch.float16: ("<f2", None),
                     torch.float32: ("<f4", None), torch.uint8: ("|u1", None),
                     torch.int8: ("|i1", None), torch.int32: ("<i4", None)}[dtype]

    class _Blob:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                    "data": (ptr, False), "version": 3, "strides": None}

    t = torch.as_tensor(_Blob(), device=f"cuda:{device}")
    return t.view(view) if view is not None else t


class ColParallelW4A16:
    """Column-parallel W4A16 linear with the fused all-gather.

    Every rank holds the full activations x [M, K] (bf16) and its weight shard
    (packed u8 [N/R, K/2], fp16 scales [N/R, K/gs]); ``__call__`` returns the
    full bf16 output [M, N] in this rank's shared buffer, identical on every
    rank once the call returns (the stream-ordered barrier is part of it)."""

    def __init__(self, M: int, N: int, K: int, group_size: int = 128, group=None, store: str = "peer"):
        """store: "peer" -- the epilogue TMA-stores each tile into every rank's
        buffer (CUDA IPC mappings), once per rank; "nvls" -- it stores each
        tile once through the NVSwitch's multicast (kc_gemm_w4a16_allgather_mc
        on a symmetric buffer), which writes it into every rank's copy
        (RuntimeError where the platform has no multicast)."""
        if store not in ("peer", "nvls"):
            raise ValueError("store must be 'peer' or 'nvls'")
        self.store = store
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.M, self.N, self.K, self.gs = M, N, K, group_size
        self.n_shard = N // self.world
        shard_range(N, self.world, self.rank)  # validates the split
        self.barrier = PeerBarrier(group)
        if store == "nvls":
            self.symm = SymmetricBuffer((M, N), torch.bfloat16, group)
            self.out = self.symm.local
            return
        self.out_bufs = PeerBuffers(M * N * 2, group)
        self.out = self.out_bufs.local((M, N), torch.bfloat16)
        self._outs = (ctypes.c_void_p * self.world)(*self.out_bufs.ptrs)

    def launch(self, x: torch.Tensor, packed_shard: torch.Tensor, scales_shard: torch.Tensor) -> None:
        """The fused GEMM alone (no barrier): for timing and for callers that
        synchronize the ranks themselves."""
        check_col_parallel_w4a16(self.M, self.K, self.n_shard, self.gs, x, packed_shard, scales_shard)
        if self.store == "nvls":
            check(lib().kc_gemm_w4a16_allgather_mc(
                ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(packed_shard.data_ptr()),
                ctypes.c_void_p(scales_shard.data_ptr()), ctypes.c_void_p(self.symm.multicast_ptr),
                self.world, self.rank, self.M, self.n_shard, self.K, self.gs, _stream()))
            return
        check(lib().kc_gemm_w4a16_allgather(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(packed_shard.data_ptr()),
            ctypes.c_void_p(scales_shard.data_ptr()), self._outs, self.world, self.rank, self.M,
            self.n_shard, self.K, self.gs, _stream()))

    def __call__(self, x, packed_shard, scales_shard, entry_barrier: bool = True) -> torch.Tensor:
        """entry_barrier: wait until no rank still reads the previous result
        before the peers overwrite it; a caller whose ranks do nothing with the
        output between calls (e.g. back-to-back calls, each ending in the exit
        barrier) may skip it."""
        if entry_barrier:
            self.barrier()
        self.launch(x, packed_shard, scales_shard)
        self.barrier()
        return self.out

    def close(self) -> None:
        torch.cuda.synchronize()
        self.barrier.close()
        if self.store == "nvls":
            self.symm.close()
            return
        self.out_bufs.close()


class RowParallelFP8:
    """Row-parallel FP8 linear: each rank's K-shard partial, summed in bf16
    into every rank's [M, N] output.

    Every rank holds its K shard of the activation and weight codes and the
    full-row scales; ``__call__`` returns this rank's [M, N] bf16 output
    buffer (the same on every rank).  ``reduce`` picks the sum:
    "fused" -- kc_gemm_fp8_allreduce, the sum inside the GEMM's epilogue
    (partial tiles to the rank owning their rows over NVLink, the owner's sum
    to every rank), between two peer barriers; "fused_nvls" --
    kc_gemm_fp8_allreduce_mc, the same with the owner summing the ranks'
    copies in the NVSwitch (multimem) on a symmetric buffer; "nvls" -- kc_allreduce_bf16_nvls
    in the NVSwitch per row block under the next block's GEMM; "peer" --
    kc_gemm_fp8 then kc_allreduce_bf16_peer between peer barriers; "nccl" --
    one NCCL all-reduce; "overlap" -- NCCL per row block."""

    def __init__(self, M: int, N: int, group=None, reduce: str = "peer", chunks: int = 4,
                 comm_sms: int = 16):
        if reduce not in ("peer", "nccl", "overlap", "nvls", "fused", "fused_nvls"):
            raise ValueError("reduce must be 'peer', 'nccl', 'overlap', 'nvls', 'fused' or 'fused_nvls'")
        self.chunks, self.comm_sms = chunks, comm_sms
        self.reduce = reduce
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.M, self.N = M, N
        if (M * N) % (8 * self.world):
            raise ValueError("M * N must be a multiple of 8 * world")
        self.barrier = PeerBarrier(group)
        if reduce in ("fused", "fused_nvls"):
            # kc_gemm_fp8_allreduce(_mc): the sum in the GEMM's epilogue
            R = self.world
            if R < 2 or M % (128 * R) or N % 256:
                raise ValueError("the fused sum needs 2+ ranks, M % (128 * ranks) == 0 and N % 256 == 0")
            per = (M // 128 // R) * (N // 256)
            self.flag_bufs = PeerBuffers((R - 1) * per * 4, group)
            self._flags = (ctypes.c_void_p * R)(*self.flag_bufs.ptrs)
            self.epoch = 0
            if reduce == "fused_nvls":
                self.symm = SymmetricBuffer((M, N), torch.bfloat16, group)
                self.out = self.symm.local
                self.flag_bufs.local(((R - 1) * per,), torch.int32).zero_()
                torch.cuda.synchronize()
                dist.barrier(group=group)
                return
            self.out_bufs = PeerBuffers(M * N * 2, group)
            self.recv_bufs = PeerBuffers((R - 1) * (M // R) * N * 2, group)
            self.flag_bufs.local(((R - 1) * per,), torch.int32).zero_()
            torch.cuda.synchronize()
            dist.barrier(group=group)          # every flag array is zero before first use
            self.out = self.out_bufs.local((M, N), torch.bfloat16)
            self._outs = (ctypes.c_void_p * R)(*self.out_bufs.ptrs)
            self._recvs = (ctypes.c_void_p * R)(*self.recv_bufs.ptrs)
            return
        if reduce == "nvls":
            # one symmetric bf16 buffer: the GEMM writes this rank's partial
            # into its own copy, the switch sums the copies in place
            self.symm = SymmetricBuffer((M, N), torch.bfloat16, group)
            self.out = self.symm.local
            self.comm = torch.cuda.Stream()
            self._events = []
            return
        self.part_bufs = PeerBuffers(M * N * 2, group)
        self.out_bufs = PeerBuffers(M * N * 2, group)
        self.partial = self.part_bufs.local((M, N), torch.bfloat16)
        self.out = self.out_bufs.local((M, N), torch.bfloat16)
        self._parts = (ctypes.c_void_p * self.world)(*self.part_bufs.ptrs)
        self._outs = (ctypes.c_void_p * self.world)(*self.out_bufs.ptrs)

    def __call__(self, a_codes_shard, sa, w_codes_shard, sw, entry_barrier: bool = True) -> torch.Tensor:
        """entry_barrier: wait until no rank still reads the previous call's
        partials or output; back-to-back calls whose ranks touch neither in
        between may skip it (the previous exit barrier orders them)."""
        check_row_parallel_fp8(self.M, self.N, a_codes_shard, sa, w_codes_shard, sw)
        Kr = a_codes_shard.shape[1]
        l = lib()
        if self.reduce == "nccl":   # GEMM into the local output, NCCL sums in place
            return row_parallel_fp8(a_codes_shard, sa, w_codes_shard, sw, self.out, self.group)
        if self.reduce == "overlap":   # row blocks: block i's all-reduce under block i+1's GEMM
            return row_parallel_fp8_overlap(a_codes_shard, sa, w_codes_shard, sw, self.out,
                                            self.chunks, self.comm_sms, self.group)
        if self.reduce == "nvls":
            return self._nvls(a_codes_shard, sa, w_codes_shard, sw, Kr, entry_barrier)
        if self.reduce in ("fused", "fused_nvls"):
            # the ranks' GEMMs start together (the flag waits are bounded), and
            # every sum is in every output after the exit barrier
            self.barrier()
            self.epoch += 1
            if self.reduce == "fused_nvls":
                check(l.kc_gemm_fp8_allreduce_mc(
                    ctypes.c_void_p(a_codes_shard.data_ptr()), ctypes.c_void_p(sa.data_ptr()),
                    ctypes.c_void_p(w_codes_shard.data_ptr()), ctypes.c_void_p(sw.data_ptr()),
                    ctypes.c_void_p(self.out.data_ptr()), ctypes.c_void_p(self.symm.multicast_ptr),
                    self._flags, self.world, self.rank, self.epoch, self.M, self.N, Kr,
                    self.barrier.timeout_ns, _stream()))
                self.barrier()
                return self.out
            check(l.kc_gemm_fp8_allreduce(
                ctypes.c_void_p(a_codes_shard.data_ptr()), ctypes.c_void_p(sa.data_ptr()),
                ctypes.c_void_p(w_codes_shard.data_ptr()), ctypes.c_void_p(sw.data_ptr()),
                self._outs, self._recvs, self._flags, self.world, self.rank, self.epoch, self.M,
                self.N, Kr, self.barrier.timeout_ns, _stream()))
            self.barrier()
            return self.out
        if entry_barrier:
            self.barrier()
        check(l.kc_gemm_fp8(ctypes.c_void_p(a_codes_shard.data_ptr()), ctypes.c_void_p(sa.data_ptr()),
                            ctypes.c_void_p(w_codes_shard.data_ptr()), ctypes.c_void_p(sw.data_ptr()),
                            ctypes.c_void_p(self.partial.data_ptr()), 0, self.M, self.N, Kr, self.N,
                            _stream()))
        self.barrier()      # every partial is complete
        check(l.kc_allreduce_bf16_peer(self._parts, self._outs, self.world, self.rank,
                                       self.M * self.N, _stream()))
        self.barrier()      # every slice is in every output
        return self.out

    def _nvls(self, a, sa, w, sw, Kr, entry_barrier):
        """Row blocks of the output: block i's GEMM on the current stream (on
        all but comm_sms SMs when there is more than one block), then on the
        comm stream a peer barrier (block i complete on every rank) and the
        in-switch sum of block i, under block i+1's GEMM; a last barrier on
        the comm stream (every slice in every copy), which the current
        stream waits for."""
        l = lib()
        M, N = self.M, self.N
        chunks = max(1, min(self.chunks, (M + 127) // 128))
        rows = -(-M // chunks)
        rows = -(-rows // 128) * 128                 # whole 128-row tiles per block
        sms = torch.cuda.get_device_properties(self.out.device).multi_processor_count
        gemm_ctas = sms if chunks == 1 else max(1, sms - self.comm_sms)
        comm_ctas = 0 if chunks == 1 else 8 * self.comm_sms
        main = torch.cuda.current_stream()
        if entry_barrier:
            self.barrier()
        self.comm.wait_stream(main)
        mc = self.symm.multicast_ptr
        for m0 in range(0, M, rows):
            mc_rows = min(rows, M - m0)
            check(l.kc_gemm_fp8_ctas(ctypes.c_void_p(a[m0:].data_ptr()), ctypes.c_void_p(sa[m0:].data_ptr()),
                                     ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(sw.data_ptr()),
                                     ctypes.c_void_p(self.out[m0:].data_ptr()), 0, mc_rows, N, Kr, N,
                                     gemm_ctas, _stream()))
            ev = torch.cuda.Event()
            ev.record(main)
            with torch.cuda.stream(self.comm):
                self.comm.wait_event(ev)
                self.barrier()                       # block complete on every rank
                check(l.kc_allreduce_bf16_nvls(ctypes.c_void_p(mc + 2 * m0 * N), self.world, self.rank,
                                               mc_rows * N, comm_ctas, _stream()))
        with torch.cuda.stream(self.comm):
            self.barrier()                           # every slice is in every copy
        main.wait_stream(self.comm)
        return self.out

    def close(self) -> None:
        torch.cuda.synchronize()
        self.barrier.close()
        if self.reduce == "nvls":
            self.symm.close()
            return
        if self.reduce == "fused_nvls":
            self.symm.close()
            self.flag_bufs.close()
            return
        if self.reduce == "fused":
            self.out_bufs.close()
            self.recv_bufs.close()
            self.flag_bufs.close()
            return
        self.part_bufs.close()
        self.out_bufs.close()


def row_parallel_fp8(a_codes_shard: torch.Tensor, sa: torch.Tensor, w_codes_shard: torch.Tensor,
                     sw: torch.Tensor, out: torch.Tensor, comm_group=None) -> torch.Tensor:
    """Row-parallel FP8 linear: out [M, N] bf16 = sum over ranks of
    (a_shard . w_shard^T) * sa[m] * sw[n], the partial of this rank computed by
    kc_gemm_fp8 into `out` and summed in place by an NCCL all-reduce."""
    M, Kr = a_codes_shard.shape
    N = w_codes_shard.shape[0]
    check_row_parallel_fp8(M, N, a_codes_shard, sa, w_codes_shard, sw)
    if tuple(out.shape) != (M, N) or out.dtype != torch.bfloat16 or out.stride(1) != 1 or not out.is_cuda:
        raise ValueError(f"out: expected a CUDA bf16 [{M}, {N}] tensor with unit column stride")
    check(lib().kc_gemm_fp8(ctypes.c_void_p(a_codes_shard.data_ptr()), ctypes.c_void_p(sa.data_ptr()),
                            ctypes.c_void_p(w_codes_shard.data_ptr()), ctypes.c_void_p(sw.data_ptr()),
                            ctypes.c_void_p(out.data_ptr()), 0, M, N, Kr, out.stride(0), _stream()))
    dist.all_reduce(out, group=comm_group)
    return out


def row_parallel_fp8_overlap(a_codes_shard: torch.Tensor, sa: torch.Tensor,
                             w_codes_shard: torch.Tensor, sw: torch.Tensor, out: torch.Tensor,
                             chunks: int = 4, comm_sms: int = 16, comm_group=None) -> torch.Tensor:
    """row_parallel_fp8 with the reduction overlapped: the M rows run as
    `chunks` GEMMs, and each finished row block's bf16 partial is summed by an
    NCCL all-reduce (on NCCL's own stream, ordered after that block's GEMM)
    while the next block's GEMM computes.  The GEMMs run on all but comm_sms
    SMs, which stay free for the collective; the current stream waits for
    every all-reduce before the call returns.  Same result as
    row_parallel_fp8, block by block."""
    M, Kr = a_codes_shard.shape
    N = w_codes_shard.shape[0]
    check_row_parallel_fp8(M, N, a_codes_shard, sa, w_codes_shard, sw)
    if tuple(out.shape) != (M, N) or out.dtype != torch.bfloat16 or not out.is_contiguous() or not out.is_cuda:
        raise ValueError(f"out: expected a contiguous CUDA bf16 [{M}, {N}] tensor")
    chunks = max(1, min(chunks, (M + 127) // 128))
    rows = -(-M // chunks)
    rows = -(-rows // 128) * 128                # whole 128-row tiles per block
    ctas = max(1, torch.cuda.get_device_properties(out.device).multi_processor_count - comm_sms)
    works = []
    for m0 in range(0, M, rows):
        mc = min(rows, M - m0)
        a = a_codes_shard[m0:m0 + mc]
        o = out[m0:m0 + mc]
        check(lib().kc_gemm_fp8_ctas(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(sa[m0:].data_ptr()),
                                     ctypes.c_void_p(w_codes_shard.data_ptr()),
                                     ctypes.c_void_p(sw.data_ptr()), ctypes.c_void_p(o.data_ptr()), 0,
                                     mc, N, Kr, N, ctas, _stream()))
        works.append(dist.all_reduce(o, group=comm_group, async_op=True))
    for w in works:
        w.wait()
    return out


def shard_w4_rows(packed: torch.Tensor, scales: torch.Tensor, world: int, rank: int):
    """Rows [r*N/R, (r+1)*N/R) of a W4 matrix [N, K] (packed u8 [N, K/2],
    scales [N, K/gs]): the weight shard of a column-parallel linear."""
    b, e = shard_range(packed.shape[0], world, rank)
    return packed[b:e].contiguous(), scales[b:e].contiguous()


def shard_w4_cols(packed: torch.Tensor, scales: torch.Tensor, group_size: int, world: int, rank: int):
    """Columns [r*K/R, (r+1)*K/R) of a W4 matrix [N, K]: the weight shard of a
    row-parallel linear.  K/R must be a multiple of the group size, so each
    shard keeps whole scale groups (packed bytes hold two k each)."""
    K = packed.shape[1] * 2
    b, e = shard_range(K, world, rank)
    if (e - b) % group_size:
        raise ValueError(f"K shard {e - b} is not a multiple of the group size {group_size}")
    return (packed[:, b // 2:e // 2].contiguous(),
            scales[:, b // group_size:e // group_size].contiguous())


class MLPBlockW4A16:
    """The reference's MLP block on GPTQ W4 weights, tensor parallel.

    x [M, H] bf16 is replicated.  Rank r holds rows [r*I/R, (r+1)*I/R) of the
    up projection W1 [I, H] (``shard_w4_rows``) and the same columns of the
    down projection W2 [H, I] (``shard_w4_cols``).  ``__call__`` computes
    h_r = gelu_quick(x . W1_r^T) with the activation in the GEMM epilogue
    (bf16, [M, I/R]), the partial y_r = h_r . W2_r^T in fp32, and sums the
    partials with one NCCL all-reduce; every rank returns y [M, H] fp32.  The
    reference's block runs the same chain (tensor_parallel.py:150-172:
    col_parallel_linear, a numpy GELU, row_parallel_linear, ring_allreduce) in
    fp32 with the activation as a separate pass.  With one process (or no
    process group) it is the plain two-GEMM block."""

    def __init__(self, M: int, H: int, I: int, group_size: int = 128, act: str = "gelu_quick",
                 group=None):
        if act not in ("gelu_quick", "none"):
            raise ValueError("act must be 'gelu_quick' or 'none'")
        self.act = kc_lib.KC_ACT_GELU_QUICK if act == "gelu_quick" else kc_lib.KC_ACT_NONE
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        self.M, self.H, self.I, self.gs = M, H, I, group_size
        b, e = shard_range(I, self.world, self.rank)
        self.i_shard = e - b
        if self.i_shard % group_size or self.i_shard % 64:
            raise ValueError(f"I/R = {self.i_shard} must be a multiple of 64 and of the group size")
        self.h = torch.empty(M, self.i_shard, dtype=torch.bfloat16, device="cuda")
        self.y = torch.empty(M, H, dtype=torch.float32, device="cuda")

    def launch(self, x, w1_packed, w1_scales, w2_packed, w2_scales) -> None:
        """Both GEMMs of this rank (no collective): for timing."""
        check_mlp_block_w4a16(self.M, self.H, self.i_shard, self.gs, x, w1_packed, w1_scales,
                              w2_packed, w2_scales)
        l = lib()
        check(l.kc_gemm_w4a16_act(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w1_packed.data_ptr()),
            ctypes.c_void_p(w1_scales.data_ptr()), ctypes.c_void_p(self.h.data_ptr()), 0, self.M,
            self.i_shard, self.H, self.gs, self.i_shard, self.act, _stream()))
        check(l.kc_gemm_w4a16(
            ctypes.c_void_p(self.h.data_ptr()), ctypes.c_void_p(w2_packed.data_ptr()),
            ctypes.c_void_p(w2_scales.data_ptr()), ctypes.c_void_p(self.y.data_ptr()), 1, self.M,
            self.H, self.i_shard, self.gs, self.H, _stream()))

    def __call__(self, x, w1_packed, w1_scales, w2_packed, w2_scales) -> torch.Tensor:
        self.launch(x, w1_packed, w1_scales, w2_packed, w2_scales)
        if self.world > 1:
            dist.all_reduce(self.y, group=self.group)
        return self.y
