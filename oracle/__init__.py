"""CPU oracle for the hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may import this
package, and only as the checker or the timed CPU baseline; the product path (libknx.so and the
modules under knivesysl-diffusion-xe_b200/kernels) never calls into it.

Each function restates the reference's algorithm and cites the reference file:line it follows
(paths inside the reference project).  Parity is pinned by tests/golden/*.npz, produced from the
reference's own code (its torch functions and its Triton kernels run by Triton's CPU interpreter)
by tests/golden/make_golden.py, and by the published Philox4x32-10 known-answer vectors.
"""
