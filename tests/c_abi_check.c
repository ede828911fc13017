/* Compiled by tests/test_c_abi.py with the system C compiler against
 * include/lfm_cuda.h and liblfm2_b200.so: prints the layout of the ABI's
 * structs and the status of the entry points that need no GPU. */
#include <stddef.h>
#include <stdio.h>

#include "lfm_cuda.h"

#define FIELD(T, f) printf(#T " " #f " %zu %zu\n", offsetof(T, f), sizeof(((T*)0)->f))

int main(int argc, char** argv) {
  printf("size lfm_hparams %zu\n", sizeof(lfm_hparams));
  FIELD(lfm_hparams, dim);
  FIELD(lfm_hparams, heads);
  FIELD(lfm_hparams, head_dim);
  FIELD(lfm_hparams, n_layers);
  FIELD(lfm_hparams, vocab);
  FIELD(lfm_hparams, n_expert);
  FIELD(lfm_hparams, n_used);
  FIELD(lfm_hparams, expert_ff);
  FIELD(lfm_hparams, n_ff);
  FIELD(lfm_hparams, dense_lead);
  FIELD(lfm_hparams, conv_l_cache);
  FIELD(lfm_hparams, eos);
  FIELD(lfm_hparams, eps);
  FIELD(lfm_hparams, rope_theta);
  FIELD(lfm_hparams, kv_heads);
  printf("size lfm_counters %zu\n", sizeof(lfm_counters));
  FIELD(lfm_counters, kernel_launches);
  FIELD(lfm_counters, gpu_argmax);
  FIELD(lfm_counters, graph_replays);
  FIELD(lfm_counters, graph_captures);
  FIELD(lfm_counters, prefill_tokens);
  FIELD(lfm_counters, expert_grouped_launches);
  lfm_hparams hp;
  lfm_status st = lfm_model_inspect(argc > 1 ? argv[1] : "/nonexistent/model.gguf", &hp);
  printf("inspect %d %s\n", (int)st, lfm_global_error());
  printf("q6k_device_bytes %zu\n", lfm_q6k_device_bytes(2048, 2048));
  return 0;
}
