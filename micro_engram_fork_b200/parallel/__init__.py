"""Multi-GPU substrate: symmetric peer buffers (CUDA IPC over NVLink), the row store of the
row-sharded engram tables, and the P2P collectives used on the hot paths."""
