"""Native data plane: column store (C++), TCP server/client, gates, ledger, adapter."""

from .client import BatchMeta, Columns, LocalClient, RemoteClient, connect

__all__ = ["BatchMeta", "Columns", "LocalClient", "RemoteClient", "connect"]
