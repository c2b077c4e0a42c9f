/* sizeof and field offsets of the structs of qmoe.h, as "struct field offset"
 * lines ("struct - size" for the size), for comparison with the ctypes mirrors. */
#include <stddef.h>
#include <stdio.h>

#include "qmoe.h"

#define S(T) printf(#T " - %zu\n", sizeof(T))
#define F(T, f) printf(#T " " #f " %zu\n", offsetof(T, f))

int main(void) {
    S(qmoe_err);
    S(qmoe_config);
    F(qmoe_config, pool_bytes); F(qmoe_config, policy); F(qmoe_config, ep_world);
    S(qmoe_q4);
    S(qmoe_layer_weights);
    F(qmoe_layer_weights, logit_bias); F(qmoe_layer_weights, gate); F(qmoe_layer_weights, sh_down);
    S(qmoe_cache_stats);
    F(qmoe_cache_stats, hot);
    S(qmoe_stats);
    F(qmoe_stats, expert_wait_seconds); F(qmoe_stats, forward_seconds); F(qmoe_stats, routed_hits);
    F(qmoe_stats, prefetch_wasted); F(qmoe_stats, expert_waves);
    S(qmoe_hc_weights);
    F(qmoe_hc_weights, norm); F(qmoe_hc_weights, down_bf16); F(qmoe_hc_weights, up); F(qmoe_hc_weights, inject);
    S(qmoe_token_args);
    F(qmoe_token_args, x); F(qmoe_token_args, x_dtype); F(qmoe_token_args, out);
    F(qmoe_token_args, shared_slot);
    S(qmoe_synth_size);
    F(qmoe_synth_size, sh_down_sb);
    S(qmoe_tensor_info);
    F(qmoe_tensor_info, shape); F(qmoe_tensor_info, nbytes); F(qmoe_tensor_info, file);
    F(qmoe_tensor_info, offset);
    S(qmoe_io_stats);
    F(qmoe_io_stats, read_seconds);
    return 0;
}
