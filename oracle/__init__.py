"""CPU oracle for MhcPre -- test infrastructure only.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use this
package, and only as the checker.  The product path (``mhcpre_review_b200``) never
imports it and has no CPU fallback.
"""
