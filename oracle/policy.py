"""Migration-policy oracle: strict remote/local ratio arithmetic and commit semantics.

Restates ``limit_pages`` (V/nvlink_migration_latency/launch_large_20261031_r2/code/backend.py:23-25),
``budget`` (final/cooperative_4gpu/code/peer/policy.py:42-46), the restore count of
``repair_active_ratio`` (peer/policy.py:107-110) and the page-table switch of
``commit`` (peer/policy.py:90-92).
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
from __future__ import annotations


def limit_pages(local: int, remote: int, numerator: int = 599, denominator: int = 10000) -> int:
    """Largest m with denominator*(remote+m) < numerator*(local-m), strictly, in integers."""
    return max(0, (numerator * local - denominator * remote - 1) // (denominator + numerator))


def budget(local: int, remote: int, peer_free: int, residents: int, numerator: int, denominator: int) -> int:
    return min(limit_pages(local, remote, numerator, denominator), peer_free, residents)


def strict_ok(local: int, remote: int, numerator: int, denominator: int) -> bool:
    return remote == 0 or denominator * remote < numerator * local


def repair_count(local: int, remote: int, numerator: int, denominator: int) -> int:
    """Slots to bring back so the strict bound holds again (0 if it already holds)."""
    if not remote or denominator * remote < numerator * local:
        return 0
    return (denominator * remote - numerator * local) // (numerator + denominator) + 1


def commit_tables(tier, slot, req_to_token, rid, pos, target) -> None:
    """Page-table switch of a committed migration: remote tier, supplier slot, req_to_token 0."""
    for r, p, t in zip(rid, pos, target):
        tier[r, p] = 1
        slot[r, p] = t
        req_to_token[r, p] = 0
