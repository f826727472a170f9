"""kvmix: FP8 and NVFP4 MLA rows in one page-id space (`kv-cache-4bit/kvmix-mixed-precision/kvmix_core.py:1-40`).

Page ids [0, P8) address the FP8 pool (576-byte rows), ids [P8, P8 + P4) the NVFP4 pool (352-byte rows), so a page
table entry alone says where a row lives.  Requests are placed by length: sequences that will stay below the
threshold (default 262,144 tokens, `kvmix_core.py:17-20`) start in FP8 (more precise), longer ones in NVFP4; when a
request grows past the threshold its pages are promoted: rows re-quantized FP8 -> NVFP4 into freshly allocated FP4
pages and the FP8 pages freed (`promote_request`, `kvmix_core.py:525`).  When the preferred pool is full the other one
serves the allocation (cross-pool fallback, `kvmix_core.py:17-22`).  Every page of one request lives in one pool, so
attention runs one sparse-MLA launch per format over the tokens of the requests in that pool.

Promotion goes through the same NVFP4 writer kernel as fresh tokens (scale rule and nibble order unchanged); on a
GPU it is enqueued on the forward stream, so it is ordered with the step that reads the promoted rows.
"""
from __future__ import annotations

from typing import Optional

import torch

from ..ops import formats as F
from ..ops import kvcache as K

PAGE = 64
DEFAULT_THRESHOLD = 262144


class PoolExhausted(RuntimeError):
    pass


class KVMixAllocator:
    def __init__(self, pages_fp8: int, pages_fp4: int, threshold: int = DEFAULT_THRESHOLD):
        self.P8, self.P4, self.threshold = pages_fp8, pages_fp4, threshold
        self.free8 = list(range(pages_fp8 - 1, -1, -1))
        self.free4 = list(range(pages_fp8 + pages_fp4 - 1, pages_fp8 - 1, -1))
        self.fallbacks = 0

    def is_fp4(self, page: int) -> bool:
        return page >= self.P8

    def local(self, page: int) -> int:
        """Page index inside its own pool."""
        return page - self.P8 if page >= self.P8 else page

    def preferred(self, total_len: int) -> str:
        return "nvfp4" if total_len >= self.threshold else "fp8"

    def alloc(self, n: int, fmt: str, fallback: bool = True) -> list:
        """n pages of format `fmt` (the other pool when it is short and `fallback`)."""
        first, other = (self.free8, self.free4) if fmt == "fp8" else (self.free4, self.free8)
        if len(first) >= n:
            return [first.pop() for _ in range(n)]
        if fallback and len(other) >= n:
            self.fallbacks += 1
            return [other.pop() for _ in range(n)]
        raise PoolExhausted(f"{n} pages of {fmt} (free fp8 {len(self.free8)}, fp4 {len(self.free4)})")

    def release(self, pages) -> None:
        for p in pages:
            (self.free4 if self.is_fp4(p) else self.free8).append(p)

    @property
    def free_tokens(self) -> int:
        return PAGE * (len(self.free8) + len(self.free4))


class KVMixPools:
    """One layer's FP8 + NVFP4 latent pools addressed by kvmix page ids."""

    def __init__(self, alloc: KVMixAllocator, device):
        self.alloc = alloc
        self.fp8 = torch.zeros(alloc.P8 * PAGE, F.MLA_FP8_ROW_BYTES, dtype=torch.uint8, device=device)
        self.fp4 = torch.zeros(alloc.P4 * PAGE, F.MLA_ROW_BYTES, dtype=torch.uint8, device=device)

    def rows_of(self, page: int) -> tuple[torch.Tensor, int]:
        pool = self.fp4 if self.alloc.is_fp4(page) else self.fp8
        return pool, self.alloc.local(page) * PAGE

    def write(self, nope: torch.Tensor, rope: torch.Tensor, pages: list, pos: torch.Tensor) -> None:
        """Write latents of positions `pos` of a request whose pages are `pages` (one pool per request)."""
        fp4 = self.alloc.is_fp4(pages[0])
        pool = self.fp4 if fp4 else self.fp8
        base = torch.tensor([self.alloc.local(p) * PAGE for p in pages], device=pos.device)
        slot = base[pos // PAGE] + pos % PAGE
        K.mla_write(nope, rope, slot.int(), pool)


class KVMixRequest:
    """Per-request placement state: pages in one pool, promoted when the sequence crosses the threshold."""

    def __init__(self, alloc: KVMixAllocator, total_len_hint: int):
        self.alloc = alloc
        self.fmt = alloc.preferred(total_len_hint)
        self.pages: list = []
        self.length = 0

    def ensure(self, new_len: int, pools: Optional[list] = None) -> bool:
        """Grow to new_len tokens; returns True when this call promoted the request to NVFP4 (pools: every layer's
        KVMixPools, re-quantized together)."""
        promoted = False
        if self.fmt == "fp8" and new_len >= self.alloc.threshold and self.pages and not self.alloc.is_fp4(
                self.pages[0]):
            if pools is None:
                raise ValueError("promotion needs the pools")
            new = self.alloc.alloc(len(self.pages), "nvfp4", fallback=False)   # one id set for every layer
            for p in pools:
                _copy_promote(p, self.pages, new, self.length)
            self.alloc.release(self.pages)
            self.pages, self.fmt, promoted = new, "nvfp4", True
        need = -(-new_len // PAGE) - len(self.pages)
        if need > 0:
            fmt = "nvfp4" if (self.pages and self.alloc.is_fp4(self.pages[0])) else self.fmt
            got = self.alloc.alloc(need, fmt, fallback=not self.pages)
            self.pages += got
            if self.alloc.is_fp4(got[0]):
                self.fmt = "nvfp4"
        self.length = max(self.length, new_len)
        return promoted

    def free(self) -> None:
        self.alloc.release(self.pages)
        self.pages = []


def _copy_promote(pools: KVMixPools, src_pages: list, dst_pages: list, n_tokens: int) -> None:
    """Re-quantize the first n_tokens rows of FP8 pages into NVFP4 pages (`promote_rows` of the reference)."""
    for j, (src, dst) in enumerate(zip(src_pages, dst_pages)):
        n = min(PAGE, n_tokens - j * PAGE)
        if n <= 0:
            break
        s0 = pools.alloc.local(src) * PAGE
        lat = F.mla_fp8_row_dequantize(pools.fp8[s0:s0 + n]).to(torch.bfloat16)   # E4M3 values are exact in bf16
        d0 = pools.alloc.local(dst) * PAGE
        slot = torch.arange(d0, d0 + n, dtype=torch.int32, device=lat.device)
        K.mla_write(lat[:, :F.MLA_NOPE].contiguous(), lat[:, F.MLA_NOPE:].contiguous(), slot, pools.fp4)


def capacity_gain(pages_fp8_equivalent_bytes: int, frac_fp4: float) -> float:
    """Tokens held in a fixed byte budget when a fraction of tokens is stored as NVFP4 instead of FP8."""
    b8, b4 = F.MLA_FP8_ROW_BYTES, F.MLA_ROW_BYTES
    per_tok = (1 - frac_fp4) * b8 + frac_fp4 * b4
    return (pages_fp8_equivalent_bytes / per_tok) / (pages_fp8_equivalent_bytes / b8)


class KVMixPageSpace:
    """The kvmix id space as the page allocator the MLA runner and its requests use (`free`, `used`, `alloc`,
    `release`, `num_pages`), with one pool per request: `view(fmt)` is an allocator drawing only from that pool, so a
    request's pages never straddle the formats (its tokens are served by one sparse-attention launch).  Page 0 is
    reserved like the plain allocator's dummy page (padding rows of a step read it)."""

    def __init__(self, pages_fp8: int, pages_fp4: int, threshold: int = DEFAULT_THRESHOLD):
        self.mix = KVMixAllocator(pages_fp8, pages_fp4, threshold)
        self.mix.free8.remove(0)
        self.num_pages = pages_fp8 + pages_fp4
        self.reserved = 1

    @property
    def free(self) -> int:
        return len(self.mix.free8) + len(self.mix.free4)

    @property
    def used(self) -> int:
        return self.num_pages - self.reserved - self.free

    def free_in(self, fmt: str) -> int:
        return len(self.mix.free8 if fmt == "fp8" else self.mix.free4)

    def alloc(self, n: int) -> list:
        return self.mix.alloc(n, "fp8")

    def release(self, pages) -> None:
        self.mix.release(pages)

    def view(self, fmt: str) -> "_PoolView":
        return _PoolView(self, fmt)


class _PoolView:
    def __init__(self, space: KVMixPageSpace, fmt: str):
        self.space, self.fmt = space, fmt

    @property
    def free(self) -> int:
        return self.space.free_in(self.fmt)

    def alloc(self, n: int) -> list:
        return self.space.mix.alloc(n, self.fmt, fallback=False)

    def release(self, pages) -> None:
        self.space.release(pages)
