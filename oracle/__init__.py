"""CPU oracle for the MXFP4 MoE hot path — test infrastructure only.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this
package. The product library never calls it.
"""
