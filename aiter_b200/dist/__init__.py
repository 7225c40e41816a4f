"""Multi-GPU plumbing of the path (the role of aiter/dist): process groups, the
CUDA-IPC custom and quick allreduces, EP dispatch / combine and the collective
front-ends."""
from .communication_op import (expert_parallel_all_gather, expert_parallel_all_reduce, expert_parallel_broadcast,
                               expert_parallel_gather, expert_parallel_reduce_scatter, shard_moe_weights_for_tp,
                               tensor_model_parallel_all_gather, tensor_model_parallel_all_reduce,
                               tensor_model_parallel_custom_all_gather, tensor_model_parallel_fused_allreduce_rmsnorm,
                               tensor_model_parallel_fused_allreduce_rmsnorm_quant, tensor_model_parallel_fused_moe,
                               tensor_model_parallel_gather, tensor_model_parallel_gemm_all_reduce,
                               tensor_model_parallel_reduce_scatter)
from .custom_all_reduce import CustomAllreduce
from .ep import EpAll2AllManager, EpDispatchCombineConfig, EpDispatchCombineOp
from .parallel_state import (GraphCaptureContext, GroupCoordinator, destroy_distributed_environment,
                             destroy_model_parallel, ensure_model_parallel_initialized, get_ep_group,
                             get_tensor_model_parallel_rank, get_tensor_model_parallel_world_size, get_tp_group,
                             get_world_group, graph_capture, in_the_same_node_as, init_distributed_environment,
                             init_model_parallel_group, init_world_group, initialize_model_parallel,
                             is_global_first_rank, model_parallel_is_initialized, patch_tensor_parallel_group,
                             prepare_communication_buffer_for_model, set_custom_all_reduce)
from .quick_all_reduce import QuickAllReduce, QuickReduceRegime
