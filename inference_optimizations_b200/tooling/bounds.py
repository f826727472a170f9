"""Host-side index checks before kernel launches (`EngineConfig.bounds_check`), the engine-native form of the
reference's IMA locator (`tooling/diagnostics/ima_locator.py`): instead of finding the faulting launch after an
illegal memory access, every index a step hands to a kernel is checked on the host (the staged lists exist there
already, so no device sync) and a violation raises before anything is launched, naming the tensor and entry."""
from __future__ import annotations


class BoundsError(RuntimeError):
    pass


def _range(name: str, values, lo: int, hi: int, allow_neg1: bool = False) -> None:
    for i, v in enumerate(values):
        if allow_neg1 and v == -1:
            continue
        if not lo <= v < hi:
            raise BoundsError(f"{name}[{i}] = {v} outside [{lo}, {hi})")


def check_gqa_pack(p, kv, rows: int) -> None:
    """Packed step of GQARunner against its KV cache: slots inside each pool, request rows inside the page tables,
    kv lengths addressable by the page-table rows, every used page-table entry a real page."""
    for kind, slots in p.slot.items():
        pages = kv.alloc[kind].num_pages if hasattr(kv.alloc[kind], "num_pages") else None
        pool = kv.pool_slots(kind) if hasattr(kv, "pool_slots") else None
        hi = pool if pool is not None else (pages * 64 if pages else 1 << 62)
        _range(f"slot[{kind}]", slots, 0, hi, allow_neg1=True)
    _range("req_idx", p.req_idx, 0, rows)
    for kind, table in kv.tables.items():
        cap = table.host.shape[1] * 64
        for i, (n, r) in enumerate(zip(p.kv_len, p.req_idx)):
            if n > cap:
                raise BoundsError(f"kv_len[{i}] = {n} > page-table capacity {cap} ({kind})")
            used = (n + 63) // 64
            row = table.host[r, :used].tolist()
            bad = [j for j, pg in enumerate(row) if pg < 0 or pg >= kv.alloc[kind].num_pages]
            if bad:
                raise BoundsError(f"page_table[{kind}][{r}][{bad[0]}] = {row[bad[0]]} not a page")


def check_mla_step(ids, pos, slot, limit, rix, kv, rows: int, vocab: int) -> None:
    _range("ids", ids, 0, vocab)
    _range("slot", slot, 0, kv.latent[0].shape[0], allow_neg1=True)
    _range("req_idx", rix, 0, rows)
    cap = kv.table.host.shape[1] * 64
    for i, (n, r) in enumerate(zip(limit, rix)):
        if n > cap:
            raise BoundsError(f"limit[{i}] = {n} > page-table capacity {cap}")
        row = kv.table.host[r, :(n + 63) // 64].tolist()
        bad = [j for j, pg in enumerate(row) if pg < 0 or pg >= kv.index[0].shape[0]]
        if bad:
            raise BoundsError(f"page_table[{r}][{bad[0]}] = {row[bad[0]]} not a page")
