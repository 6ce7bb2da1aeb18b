"""Tagged GPU buffers that can give their physical memory back and get it again at the same address.

Python side of ``csrc/runtime/vmm_alloc.cpp`` (the torch_memory_saver equivalent, reference
``axrl/ray/ray_utils.py:33-41``, ``axrl/worker/megatron_worker.py:1463-1480``).  The rollout
engine keeps its KV cache in such a buffer: it is paused (unmapped, no backup) while the trainer
needs the memory and resumed before the next rollout at the SAME virtual address, so the decode
CUDA graphs that captured its pointer stay valid.
"""

from __future__ import annotations

import torch

from axrl_b200.rollout.kv import runtime_module

_DT = {torch.bfloat16: "<V2", torch.float16: "<f2", torch.float32: "<f4", torch.uint8: "|u1", torch.int32: "<i4", torch.int64: "<i8"}


class _CudaArray:
    def __init__(self, ptr: int, shape: tuple, typestr: str) -> None:
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3, "strides": None}


class VmmBuffer:
    """A device tensor whose physical backing is owned by the tagged VMM allocator."""

    def __init__(self, shape: tuple, dtype: torch.dtype, tag: str, device: int | None = None) -> None:
        self.rt = runtime_module()
        self.tag = tag
        dev = torch.cuda.current_device() if device is None else device
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.tensor([], dtype=dtype).element_size()
        prev = self.rt.vmm_tag()
        self.rt.vmm_set_tag(tag)
        try:
            self.ptr = self.rt.vmm_malloc(nbytes, dev)
        finally:
            self.rt.vmm_set_tag(prev)
        if dtype == torch.bfloat16:  # __cuda_array_interface__ has no bf16: view int16 storage
            raw = torch.as_tensor(_CudaArray(self.ptr, (n,), "<i2"), device=f"cuda:{dev}")
            self.tensor = raw.view(torch.bfloat16).view(shape)
        else:
            self.tensor = torch.as_tensor(_CudaArray(self.ptr, tuple(shape), _DT[dtype]), device=f"cuda:{dev}")
        self.nbytes = nbytes

    def pause(self, backup: bool = False) -> int:
        torch.cuda.synchronize()
        return self.rt.vmm_pause(self.tag, backup)

    def resume(self) -> int:
        torch.cuda.synchronize()
        torch.cuda.empty_cache()  # give torch-cached memory back so the physical pages can be re-created
        return self.rt.vmm_resume(self.tag)

    def free(self) -> None:
        self.tensor = None
        self.rt.vmm_free(self.ptr)
