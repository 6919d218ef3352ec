"""Host-side callers of the transfer ops: GPU connectors and pinned allocators."""
