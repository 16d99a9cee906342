"""CPU fp32 oracle for the vision-tower hot path -- TEST INFRASTRUCTURE, not product code.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and `--impl reference`)
import this package, and only to check or time the CUDA path; nothing in strix_halo_maxx_b200/
imports it.  tower_ref.py restates moondream/gpu/md2fast.py:147-160 and is pinned against the
reference's own FastMD2._vision by tests/golden (fixtures made by tests/golden/make_golden.py,
which imports the reference read-only).  tapnext_ref.py restates the TAPNext-style step of the
BASELINE config (ViT block + RG-LRU, tapnext/npu/r9/cpuemu.py:33-47): its RG-LRU is pinned to the
reference's ssm_ref (tests/golden/make_golden_ssm.py, rglru_ref_cases.npz) and its ViT block uses
tower_ref's pinned operations, but the composition is the BASELINE simplification, which nothing in the
reference pins (the vendored TAPNext model and weights are not in the repository).  tapnextpp_ref.py
restates the full TAPNext++ block (its SSM numerics pinned to ssm_ref, the block as a whole unpinned)
and the tracking heads (pinned to the reference's Step8.heads_np).  text_ref.py, i8_ref.py and
resize_ref.py are pinned as their headers describe.
"""
