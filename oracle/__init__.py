"""CPU fp32 oracle for the vision-tower hot path -- TEST INFRASTRUCTURE, not product code.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and `--impl reference`)
import this package, and only to check or time the CUDA path; nothing in strix_halo_maxx_b200/
imports it.  tower_ref.py restates moondream/gpu/md2fast.py:147-160 and is pinned against the
reference's own FastMD2._vision by tests/golden (fixtures made by tests/golden/make_golden.py,
which imports the reference read-only).  tapnext_ref.py restates the TAPNext-style step of the
BASELINE config (ViT block + RG-LRU, tapnext/npu/r9/cpuemu.py:33-47); its parity is unpinned
because the vendored TAPNext model and weights are not in the reference repository.
"""
