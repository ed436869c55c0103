"""Symmetric buffers of the expert-parallel exchange over peer memory (NVLink).

Each rank allocates one buffer with the library (``lmoe_p2p_alloc``: cudaMalloc + a CUDA
IPC handle), the handles are all-gathered once over the expert-parallel process group, and
every rank maps its peers' buffers (``lmoe_p2p_open``).  From then on a step moves rows
with the library's kernels only (``lmoe_p2p_exchange_counts``, ``lmoe_p2p_dispatch``,
``lmoe_p2p_wait``, then ``lmoe_p2p_down_gemm`` -- the down projection whose epilogue writes
each output row into its source's slot -- or ``lmoe_p2p_send_back``): no NCCL call and no
host synchronisation, so the whole step can be captured in a CUDA graph.  This replaces the NCCL all-to-alls of
python/light_moe/distributed/expert_parallel.py:186-244 and :275-319.
"""
import ctypes

import torch
import torch.distributed as dist

from . import capi


class _DeviceSpan:
    """A raw device range exposed through __cuda_array_interface__ (int16 elements)."""

    def __init__(self, ptr: int, rows: int, cols: int):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """This rank's symmetric buffer and the device array of every rank's mapped buffer.

    Collective: every rank of ``group`` constructs it with the same geometry (``capacity_tokens``
    = the most tokens any rank passes in one step).  ``rows`` is the local rows region
    ([ep*Tc*k + S*Tc, d] bf16, the grouped GEMMs' input) and ``ret`` the returned slots
    ([Tc*k, d] bf16, the combine's input)."""

    def __init__(self, group, num_experts: int, capacity_tokens: int, top_k: int, num_shared: int, hidden: int,
                 device: torch.device):
        self.ep, self.me = group.ep_size, group.rank
        self.pg = group.group
        self.geometry = (self.ep, num_experts, int(capacity_tokens), top_k, num_shared, hidden)
        self.num_experts, self.capacity_tokens, self.top_k = num_experts, int(capacity_tokens), top_k
        self.num_shared, self.hidden = num_shared, hidden
        self.device = device
        lib = capi.lib()
        nbytes = lib.lmoe_p2p_buffer_bytes(*self.geometry)
        if nbytes == 0:
            raise ValueError(f"bad peer-exchange geometry {self.geometry}")
        rows_off, ret_off = ctypes.c_size_t(), ctypes.c_size_t()
        capi.call("lmoe_p2p_buffer_offsets", *self.geometry, ctypes.byref(rows_off), ctypes.byref(ret_off))
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(device):
            capi.call("lmoe_p2p_alloc", nbytes, ctypes.byref(ptr), handle)
        self._own = ptr.value
        self._mapped = []
        # every rank's IPC handle, gathered over the group (a one-time exchange; NCCL groups
        # gather device tensors, others host tensors)
        on_dev = dist.get_backend(self.pg) == "nccl"
        h = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device if on_dev else "cpu")
        gathered = [torch.empty_like(h) for _ in range(self.ep)]
        dist.all_gather(gathered, h, group=self.pg)
        bases = []
        with torch.cuda.device(device):
            for r in range(self.ep):
                if r == self.me:
                    bases.append(self._own)
                    continue
                raw = (ctypes.c_uint8 * 64)(*gathered[r].cpu().tolist())
                p = ctypes.c_void_p()
                capi.call("lmoe_p2p_open", raw, ctypes.byref(p))
                self._mapped.append(p.value)
                bases.append(p.value)
        self.peers = torch.tensor(bases, dtype=torch.int64, device=device)   # uint64 bits
        self.state = torch.zeros(4, dtype=torch.int32, device=device)
        Tc, k, S, d = self.capacity_tokens, top_k, num_shared, hidden
        self.routed_rows = self.ep * Tc * k
        self.rows = torch.as_tensor(_DeviceSpan(self._own + rows_off.value, self.routed_rows + S * Tc, d),
                                    device=device).view(torch.bfloat16)
        self.ret = torch.as_tensor(_DeviceSpan(self._own + ret_off.value, Tc * k, d), device=device).view(torch.bfloat16)
        epr = num_experts // self.ep
        self.seg_offsets = torch.zeros(epr + 2 + S, dtype=torch.int32, device=device)
        self.dst_base = torch.zeros(num_experts, dtype=torch.int32, device=device)
        # destinations of the fused down GEMM: every rank's ret region, then this rank's
        # shared-expert outputs [S * T, d]
        self.shared_out = torch.empty(max(S * Tc, 1), d, dtype=torch.bfloat16, device=device)
        self.dest_bases = torch.tensor([b + ret_off.value for b in bases] + [self.shared_out.data_ptr()],
                                       dtype=torch.int64, device=device)
        capi.call("lmoe_p2p_init", self.peers.data_ptr(), self.me, self.ep, num_experts, Tc, k, S, d,
                  self.state.data_ptr(), capi.stream_handle())
        torch.cuda.synchronize(device)
        dist.barrier(group=self.pg)   # every buffer is mapped before any rank writes to a peer

    def _args(self, num_tokens: int):
        return (self.peers.data_ptr(), self.me, self.ep, self.num_experts, self.capacity_tokens, self.top_k,
                self.num_shared, self.hidden, int(num_tokens), self.state.data_ptr())

    def exchange_counts(self, counts: torch.Tensor, num_tokens: int):
        capi.call("lmoe_p2p_exchange_counts", *self._args(num_tokens), counts.data_ptr(),
                  self.seg_offsets.data_ptr(), self.dst_base.data_ptr(), capi.stream_handle())

    def dispatch(self, x: torch.Tensor, sorted_idx, ids, offsets):
        if x.dtype != torch.bfloat16 or x.device != self.device or not x.is_contiguous():
            raise ValueError("the peer-memory exchange moves contiguous bf16 rows on its device "
                             "(the W4A16 GEMMs' input type)")
        T = x.shape[0]
        capi.call("lmoe_p2p_dispatch", *self._args(T), x.data_ptr() if T else None,
                  sorted_idx.data_ptr() if T else None, ids.data_ptr() if T else None,
                  offsets.data_ptr() if T else None, self.dst_base.data_ptr(), capi.stream_handle())

    def wait_rows(self, num_tokens: int):
        capi.call("lmoe_p2p_wait", *self._args(num_tokens), 1, capi.stream_handle())

    def send_back(self, out: torch.Tensor, num_tokens: int):
        capi.call("lmoe_p2p_send_back", *self._args(num_tokens), out.data_ptr(), self.seg_offsets.data_ptr(),
                  capi.stream_handle())

    def down_gemm(self, h: torch.Tensor, w2_packed: torch.Tensor, ffn_size: int, group_size: int,
                  seg_expert: torch.Tensor, num_segments: int, num_weight_matrices: int, num_tokens: int):
        """The down projection of the rows region with the return transfer fused into its
        epilogue (routed rows straight into their sources' ret slots), then the return flags."""
        capi.call("lmoe_p2p_down_gemm", *self._args(num_tokens), self._own, h.data_ptr(), ffn_size,
                  w2_packed.data_ptr(), group_size, self.seg_offsets.data_ptr(), seg_expert.data_ptr(),
                  num_segments, num_weight_matrices, self.dest_bases.data_ptr(), capi.stream_handle())

    def wait_returns(self, num_tokens: int):
        capi.call("lmoe_p2p_wait", *self._args(num_tokens), 2, capi.stream_handle())

    def error(self) -> int:
        """The device error word (0: no wait ran out of time, counts were consistent)."""
        return int(self.state[1].item())

    def close(self):
        """Collective: unmap the peers' buffers and free this rank's, after every rank's work."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.pg)
        with torch.cuda.device(self.device):
            for p in self._mapped:
                capi.call("lmoe_p2p_close", p)
            self._mapped = []
            self.rows = self.ret = None
            capi.call("lmoe_p2p_free", self._own)
        self._own = None
