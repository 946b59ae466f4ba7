"""Single-process fake world with the reference's exact semantics
(crates/mt-comm/src/mock.rs): a shared [src][dst] mailbox where the last send
wins, a recv that neither blocks nor consumes, and "collectives" that reduce
world_size copies of the caller's own data as little-endian u64 (Sum = n*x,
Product = x^n, Mean = x)."""
from .._ext import host as _host

MockCommunicator = _host().MockCommunicator

__all__ = ["MockCommunicator"]
