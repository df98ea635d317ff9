"""CPU oracle for the decode/prefill step -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs import this package.  It is the checker, never the thing measured or
shipped: the engine in tvara_b200/ has no CPU fallback and does not import it.

* ``lib()``       -- liboracle.so, the C restatement in oracle.c
* ``ref()``       -- oracle/_ref/libtvara_refshim.so, the reference's own headers
                     compiled here (absent where the reference was not built)
* ``ref_capi()``  -- oracle/_ref/libtvara_capi.so, the reference engine's C ABI
* ``reference_module(name)`` -- a module of the reference's Python package,
                     staged unchanged into oracle/_ref/python (None if absent)
* ``model.OracleModel`` -- numpy restatement of PagedModelExecutor::decode
"""

from .oracle import lib, ref, ref_capi, ref_available, reference_module, ORACLE_DIR  # noqa: F401
