"""The IR packages the parity tests and the baseline use, by tag.

Each tag maps to ``(builder name, builder kwargs)`` in
``emmy_ptx.workloads``.  PARITY cases are small enough for the CPU oracle;
they include ragged shapes (row/column counts that do not fill the last
block, a loop whose trip count differs between threads).  FULL cases are the
BASELINE configs at their full sizes.
"""

PARITY = {
    "pointwise_f32_64x256": ("pointwise_f32", dict(rows=64, cols=256)),
    "pointwise_f32_33x100": ("pointwise_f32", dict(rows=33, cols=100)),
    "pointwise_i32_64x256": ("pointwise_i32", dict(rows=64, cols=256)),
    "pointwise_i32_33x100": ("pointwise_i32", dict(rows=33, cols=100)),
    "rmsnorm_16x1024": ("rmsnorm", dict(rows=16, cols=1024)),
    "rmsnorm_5x1000": ("rmsnorm", dict(rows=5, cols=1000)),
    "softmax_8x4096": ("softmax", dict(rows=8, cols=4096)),
    "softmax_3x2052": ("softmax", dict(rows=3, cols=2052)),
    "softmax_4x16384": ("softmax", dict(rows=4, cols=16384)),
    "softmax_300x16384": ("softmax", dict(rows=300, cols=16384)),
    "colreduce_f64_256x128": ("colreduce_f64", dict(rows=256, cols=128)),
    "colreduce_f64_100x64": ("colreduce_f64", dict(rows=100, cols=64)),
    "rowsum_i32_64x1024": ("rowsum_i32", dict(rows=64, cols=1024)),
    "rowsum_i32_7x68": ("rowsum_i32", dict(rows=7, cols=68)),
    "matmul_128x128x64": ("matmul", dict(m=128, n=128, k=64)),
    "matmul_256x384x128": ("matmul", dict(m=256, n=384, k=128)),
    # four K groups of 256: the kernel's warps 2-3 split groups 1-3 themselves
    "matmul_256x256x1024": ("matmul", dict(m=256, n=256, k=1024)),
    "attention_1x2x64x128": ("attention", dict(batch=1, heads=2, seq=64, head_dim=128)),
    "attention_2x1x40x64": ("attention", dict(batch=2, heads=1, seq=40, head_dim=64)),
    "attention_noncausal_1x2x48x64": ("attention", dict(batch=1, heads=2, seq=48, head_dim=64,
                                                        causal=False)),
    # several head groups: the kernel splits groups 1.. itself (its split warp)
    "attention_2x8x256x128": ("attention", dict(batch=2, heads=8, seq=256, head_dim=128)),
    "attention_3x5x256x64": ("attention", dict(batch=3, heads=5, seq=256, head_dim=64)),
    "attention_noncausal_2x6x192x64": ("attention", dict(batch=2, heads=6, seq=192, head_dim=64,
                                                         causal=False)),
    "pointwise_zoo_16x64": ("pointwise_zoo", dict(rows=16, cols=64)),
    "pointwise_mixed_16x64": ("pointwise_mixed", dict(rows=16, cols=64)),
    "bit_ops_16x64": ("bit_ops", dict(rows=16, cols=64)),
    "bit_ops_7x36": ("bit_ops", dict(rows=7, cols=36)),
    "rowsum_f64_9x300": ("rowsum_f64", dict(rows=9, cols=300)),
    "rowsum_f64_64x512": ("rowsum_f64", dict(rows=64, cols=512)),
    "offset_copy_8x64_o1": ("offset_copy", dict(rows=8, cols=64, offset=1, pad=4)),
    "offset_copy_5x68_p2": ("offset_copy", dict(rows=5, cols=68, offset=0, pad=2)),
}

FULL = {
    "pointwise_f32_full": ("pointwise_f32", {}),
    "pointwise_i32_full": ("pointwise_i32", {}),
    "rmsnorm_full": ("rmsnorm", {}),
    "softmax_full": ("softmax", {}),
    "colreduce_f64_full": ("colreduce_f64", {}),
    "rowsum_i32_full": ("rowsum_i32", {}),
    "matmul_full": ("matmul", {}),
    "attention_full": ("attention", {}),
}

ALL = {**PARITY, **FULL}


def problem(tag):
    from emmy_ptx import workloads
    name, kw = ALL[tag]
    return workloads.build(name, **kw)
