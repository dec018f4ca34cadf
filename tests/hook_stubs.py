"""Stand-ins with the parameter lists of vLLM's prepare_nvfp4_moe_layer_for_marlin and fused_marlin_moe (vLLM 0.22,
vllm/.../marlin_utils_fp4.py and fused_moe/experts/marlin_moe.py), for testing the hook without running vLLM."""


class Reached(Exception):
    pass


def stub_prepare(layer, w13, w13_scale, w13_scale_2, w2, w2_scale, w2_scale_2, is_act_and_mul):
    raise Reached("original prepare")


def stub_fused(hidden_states, w1, w2, bias1, bias2, w1_scale, w2_scale, topk_weights, topk_ids, quant_type_id,
               apply_router_weight_on_input=False, global_num_experts=-1, activation=None, activation_func=None,
               moe_sum=None, expert_map=None, input_global_scale1=None, input_global_scale2=None, global_scale1=None,
               global_scale2=None, g_idx1=None, g_idx2=None, sort_indices1=None, sort_indices2=None, w1_zeros=None,
               w2_zeros=None, workspace=None, intermediate_cache13=None, intermediate_cache2=None, is_k_full=True,
               output=None, input_dtype=None, inplace=False, clamp_limit=None):
    raise Reached("original fused_marlin_moe")
