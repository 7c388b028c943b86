"""CPU oracle for the w8g64 qlinear / AV DiT block path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs, never by the product library.

  oracle.lib      ctypes over liboracle.so (ltx_oracle.c, the restatement)
  oracle.ref      ctypes over _ref/libref_oracle.so (the reference's own code)
  oracle.rope_np  numpy restatement of src/ltx25-rope.cc
  oracle.block_np numpy restatement of src/ltx25-block-ref.cc
"""
