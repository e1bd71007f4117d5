"""CPU checker for the B200 MoE kernels (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm import this
package.  The product library never links, loads or calls it.
"""
