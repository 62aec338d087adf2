"""Device operators of the packed-state decode path (libstepquant_b200).

``pool``       PackedStatePool and the page layout; launches the fused step
               (synchronous pools) or readout + background writeback.
``writeback``  deferred / chunked background writeback under CUDA-graph capture.
``resources``  SM-bounded writeback streams (green contexts).
``profiles``   per-batch writeback budgets.
"""
