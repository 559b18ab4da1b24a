"""KV-head tensor-parallel verify attention: each GPU holds 1/N of the KV heads, attends with them, and one NCCL
all-gather over NVLink gives every GPU the attention output of all heads.

Head split as in the reference's tensor parallelism: Qwen3Attention keeps total_heads / world query heads and
total_kv_heads / world KV heads per rank (nanovllm/models/qwen3.py:29-35), the model runner sizes each rank's
KV cache for num_key_value_heads // world heads (nanovllm/engine/model_runner.py:149), and the q/k/v weights
are chunked along the head dimension in rank order (nanovllm/layers/linear.py:92,127), so rank r holds query
heads [r*H/N, (r+1)*H/N) and KV heads [r*Hkv/N, (r+1)*Hkv/N).  Each rank's attention is the single-GPU path
(store of its K/V heads, then the tcgen05 paged kernel over its cache) with no collective; the GQA group
H/Hkv is unchanged by the split, so every (row, KV head) item still packs its 8 queries x 4 heads.

The reference follows attention with a row-parallel o_proj and an all-reduce (nanovllm/layers/linear.py:154).
This mode instead gathers the attention outputs, for a forward whose other layers are replicated:
    1. the kernel writes this rank's heads straight into chunk `rank` of a persistent [N, T, H/N, D] buffer
       (the layout NCCL's all-gather produces: rank-major, each chunk contiguous);
    2. all_gather_into_tensor in place (NCCL over NVLink / NVSwitch; 2*T*H*D*(N-1)/N bytes in per GPU);
    3. one copy interleaves the chunks into [T, H, D] (head index r*H/N + j).
Only the outputs cross GPUs: the KV cache, the dominant bytes, stays local.

exchange="peer" fuses the gather into the kernel: every rank's [T, H, D] output lives in symmetric memory
(torch.distributed._symmetric_memory: one allocation per rank, mapped into every rank's process), and the
attention kernel stores each finished tile at this rank's head offset into all N outputs (specdec_paged_
attention_multi; the peers' copies cross NVLink as plain stores while later tiles still compute).  One bounded
cross-GPU barrier kernel (specdec_peer_barrier) then orders every rank's reads after all peers' stores.  No NCCL
call and no interleave copy; the outputs alternate between two slots, so one barrier per call suffices (a rank
writes slot s again only after every peer passed the barrier that follows its use of slot s).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
from torch import nn

from . import _lib
from ._lib import check, stream_of
from .attention import Attention


def shard_heads(num_heads: int, num_kv_heads: int, world: int, rank: int) -> tuple[slice, slice]:
    """(query heads, KV heads) held by `rank` of `world`: contiguous chunks in rank order (qwen3.py:29-35,
    linear.py:92).  Raises if the heads do not split evenly or the GQA group would straddle ranks."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_kv_heads % world or num_heads % num_kv_heads:
        raise ValueError(f"{num_heads} query / {num_kv_heads} KV heads do not split over {world} ranks")
    hq, hk = num_heads // world, num_kv_heads // world
    return slice(rank * hq, (rank + 1) * hq), slice(rank * hk, (rank + 1) * hk)


def interleave_heads(gathered: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[N, T, H/N, D] rank-major chunks -> [T, H, D] with rank r's head j at head r*H/N + j."""
    N, T, Hl, D = gathered.shape
    if out is None:
        out = torch.empty(T, N * Hl, D, dtype=gathered.dtype, device=gathered.device)
    out.view(T, N, Hl, D).copy_(gathered.permute(1, 0, 2, 3))
    return out


class TPAttention(nn.Module):
    """Attention over this rank's KV heads, outputs of all heads all-gathered.

    forward(q, k, v) takes this rank's heads as the reference's Qwen3Attention hands them to its attention
    (nanovllm/models/qwen3.py, after the column-parallel qkv_proj): q [T, H/N, D] (or [T, H/N * D]), k / v
    [T, Hkv/N, D]; k_cache / v_cache are this rank's [blocks, block_size, Hkv/N, D] caches (set like the
    reference's Attention.k_cache).  Returns [T, H, D] bf16, identical on every rank.  The gather buffer is
    persistent (grown to the largest T seen), so a captured CUDA graph keeps valid pointers; NCCL calls captured
    in a graph need that graph released before the process group is destroyed.  With exchange="peer" each module
    owns one symmetric allocation (2 x max_tokens x H x D bf16 plus its arrival words) made by a collective
    rendezvous, so a model keeps one module and binds each layer's caches before that layer's call: the layers'
    calls are sequential on one stream, so the two alternating slots and the one barrier per call stay correct
    across layers."""

    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int,
                 group: dist.ProcessGroup | None = None, *, world: int | None = None, rank: int | None = None,
                 exchange: str = "nccl", max_tokens: int = 0, device: torch.device | None = None,
                 barrier_timeout_s: float = 5.0):
        """world / rank default to the process group's; giving them without a group builds one rank's module
        for ranks emulated in one process (its local() and gather_buffer() work, all_gather() needs the
        group).  exchange "nccl" (all-gather) or "peer" (stores into the peers' symmetric buffers + barrier);
        "peer" is collective at construction (every rank builds its module together) and needs max_tokens (the
        largest T of any call) and the rank's CUDA device."""
        super().__init__()
        self.group = group
        if world is None:
            world = dist.get_world_size(group) if dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world, self.rank = world, rank
        self.q_heads, self.kv_heads = shard_heads(num_heads, num_kv_heads, self.world, self.rank)
        self.num_heads, self.head_dim = num_heads, head_dim
        self.local = Attention(num_heads // self.world, head_dim, scale, num_kv_heads // self.world)
        self._buffer = torch.empty(0)
        self._retired: list[torch.Tensor] = []
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange {exchange!r}: 'nccl' or 'peer'")
        self.exchange = exchange
        if exchange == "peer":
            self._setup_peer(max_tokens, device, barrier_timeout_s)

    # ------------------------------------------------------------------------------------ peer-store exchange
    _FLAG_BYTES = 256       # 8 uint32 arrival words (one per rank), padded

    def _setup_peer(self, max_tokens: int, device: torch.device | None, timeout_s: float) -> None:
        import torch.distributed._symmetric_memory as symm_mem
        if max_tokens < 1 or device is None or device.type != "cuda":
            raise ValueError("exchange='peer' needs max_tokens >= 1 and the rank's CUDA device")
        if not dist.is_initialized() or self.world > 8:
            raise ValueError("exchange='peer' needs an initialised process group of at most 8 ranks")
        H, D = self.num_heads, self.head_dim
        self.max_tokens = max_tokens
        self._slot_bytes = max_tokens * H * D * 2
        nbytes = 2 * self._slot_bytes + self._FLAG_BYTES
        storage = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        handle = symm_mem.rendezvous(storage, self.group if self.group is not None else dist.group.WORLD)
        self._symm, self._handle = storage, handle
        ptrs = [int(p) for p in handle.buffer_ptrs]
        delta = storage.data_ptr() - ptrs[self.rank]          # 0 unless the tensor sits inside its allocation
        self._peer_ptrs = [p + delta for p in ptrs]
        self._slots = [storage[i * self._slot_bytes:(i + 1) * self._slot_bytes].view(torch.bfloat16)
                       .view(max_tokens, H, D) for i in range(2)]
        storage[2 * self._slot_bytes:].zero_()                      # this rank's arrival words
        self._epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self._err = torch.zeros(1, dtype=torch.int32, device=device)
        self._flag_ptrs = (ctypes.c_void_p * self.world)(*[p + 2 * self._slot_bytes for p in self._peer_ptrs])
        self._timeout_ns = int(timeout_s * 1e9)
        self._calls = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)                              # every rank's words are zero before use

    def peer_error(self) -> int:
        """0, or 21 when a barrier wait gave up (a peer never arrived within the timeout); synchronises.  After 21
        the ranks' barrier epochs may disagree: the module is unusable and a new one (a new rendezvous) replaces
        it."""
        return int(self._err.item())

    def _forward_peer(self, q, k, v, T: int) -> torch.Tensor:
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens: this module's symmetric buffers hold {self.max_tokens}")
        slot = self._calls % 2
        self._calls += 1
        H, D, Hl = self.num_heads, self.head_dim, self.num_heads // self.world
        offset = slot * self._slot_bytes + self.rank * Hl * D * 2      # this rank's heads in every rank's slot
        self.local.forward_to(q, k, v, [p + offset for p in self._peer_ptrs], H * D)
        check(_lib.lib().specdec_peer_barrier(self._flag_ptrs, self.world, self.rank, self._epoch.data_ptr(),
                                              self._timeout_ns, self._err.data_ptr(), stream_of(q.device)))
        return self._slots[slot][:T]

    @property
    def k_cache(self) -> torch.Tensor:
        return self.local.k_cache

    @k_cache.setter
    def k_cache(self, value: torch.Tensor) -> None:
        self.local.k_cache = value

    @property
    def v_cache(self) -> torch.Tensor:
        return self.local.v_cache

    @v_cache.setter
    def v_cache(self, value: torch.Tensor) -> None:
        self.local.v_cache = value

    def gather_buffer(self, T: int, device: torch.device) -> torch.Tensor:
        """The [N, T, H/N, D] bf16 all-gather buffer (a view of the persistent storage)."""
        Hl, D = self.num_heads // self.world, self.head_dim
        need = self.world * T * Hl * D
        if self._buffer.numel() < need or self._buffer.device != device:
            if self._buffer.numel():
                self._retired.append(self._buffer)       # a captured graph may still address it
            self._buffer = torch.empty(need, dtype=torch.bfloat16, device=device)
        return self._buffer[:need].view(self.world, T, Hl, D)

    def all_gather(self, gathered: torch.Tensor) -> torch.Tensor:
        """In-place all-gather of chunk `rank` of `gathered` into every rank's copy (no-op on one rank)."""
        if self.world > 1:
            flat = gathered.view(-1)
            dist.all_gather_into_tensor(flat, gathered[self.rank].view(-1), group=self.group)
        return gathered

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None
                ) -> torch.Tensor:
        """[T, H, D] attention output of all heads.  With exchange="peer" and no `out`, a view of this rank's
        symmetric slot, valid only until this module's next call: a peer that has passed that call's barrier
        may already be storing the call after it into the same slot.  Copy it, or pass `out`, to keep it longer."""
        T = q.numel() // ((self.num_heads // self.world) * self.head_dim)
        if self.exchange == "peer":
            result = self._forward_peer(q, k, v, T)
            return result if out is None else out.copy_(result)
        gathered = self.gather_buffer(T, q.device)
        self.local(q, k, v, out=gathered[self.rank])
        return interleave_heads(self.all_gather(gathered), out)
