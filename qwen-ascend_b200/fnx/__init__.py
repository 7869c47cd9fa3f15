"""fnx (B200 build): the W4A16 MoE expert path of qwen-ascend on sm_100a.

Drop-in modules keep the reference's ``fnx`` call signatures and ``None``-means-
unsupported convention; the compute runs in ``libfnx_b200.so`` (see ``_lib``).

    expert_gather.gather       moe_epilogue.merge       weighted_reduce.reduce
    post_ops.moe_merge         w4gemv_op.W4GemvOp
    engine.ExpW4 / DenseW8 / MoELayer   (quantised containers and the MoE layer)
    ep.ExpertParallelMoE       (experts sharded over GPUs, NCCL all-to-all)
"""
__all__ = ["expert_gather", "moe_epilogue", "weighted_reduce", "post_ops", "w4gemv_op", "engine", "synth"]
