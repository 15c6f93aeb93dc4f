"""TEST INFRASTRUCTURE -- CPU oracle of the KV-cache hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this package.  It is the checker, never the thing measured as the
product and never a fallback of the product: lattice_b200 does not import it.

Contents:
  pool_oracle   Python restatement of the reference's block allocator and
                block table (ref src/kcmm/pool.rs, src/kcmm/superblock.rs,
                src/kcmm/tiering.rs CpuSlotAllocator).
  native        ctypes access to the C restatement (kcmm_oracle.c) and to the
                reference's own kernels compiled for the host (oracle/_ref).
"""
