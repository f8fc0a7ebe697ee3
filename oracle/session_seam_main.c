/*
 * Session-seam check (test infrastructure): the reference's own prompt/session
 * state machine (FPGA_Project/software/qmap_prompt_demo/qot_session.c, compiled
 * from the reference sources by oracle/build_ref.py) driven with
 * q4gpu_run_token as its runner (qot_session_runner_fn,
 * qot_session.h:51-58).  Prints one line per token event and the stop reason,
 * so a test can compare the generated ids with the CPU oracle's greedy decode.
 *
 *   session_seam <n_layers> <vocab> <seed> <gamma_std> <max_new> <token>...
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qot_session.h"
#include "q4gpu.h"

int main(int argc, char **argv) {
  if (argc < 7) {
    fprintf(stderr, "usage: %s n_layers vocab seed gamma_std max_new token...\n", argv[0]);
    return 2;
  }
  const int n_layers = atoi(argv[1]), vocab = atoi(argv[2]);
  const unsigned long long seed = strtoull(argv[3], NULL, 10);
  const float gamma_std = (float)atof(argv[4]);
  const unsigned max_new = (unsigned)atoi(argv[5]);
  const int n_prompt = argc - 6;
  uint32_t *prompt = (uint32_t *)calloc((size_t)n_prompt, sizeof(uint32_t));
  for (int i = 0; i < n_prompt; ++i) prompt[i] = (uint32_t)strtoul(argv[6 + i], NULL, 10);

  q4gpu_model_config mc;
  memset(&mc, 0, sizeof(mc));
  mc.n_layers = n_layers;
  mc.vocab = vocab;
  mc.max_context = QOT_MAX_CONTEXT;
  mc.max_seqs = 1;
  mc.device = 0;
  q4gpu_model *gpu = NULL;
  if (q4gpu_model_create(&mc, &gpu) != Q4GPU_OK || q4gpu_model_init_synthetic(gpu, seed, 0.02f, gamma_std) != Q4GPU_OK) {
    fprintf(stderr, "model: %s\n", q4gpu_last_error());
    return 3;
  }

  qot_run_config_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.layer_start = 0;
  cfg.layer_count = (uint32_t)n_layers;
  cfg.position = 0;
  cfg.runtime_context_enable = 1;
  cfg.embedding_enable = 1;

  qot_session_t s;
  int rc = qot_session_init(&s, 0, &cfg, q4gpu_run_token, gpu);
  qot_session_options_t o;
  qot_session_default_options(&o);
  o.max_new_tokens = max_new;
  if (rc == QOT_OK) rc = qot_session_begin(&s, prompt, (uint32_t)n_prompt, &o);
  if (rc != QOT_OK) {
    fprintf(stderr, "session begin: %d\n", rc);
    return 4;
  }
  int steps = 0;
  while (!qot_session_is_terminal(&s) && steps < 4 * (n_prompt + (int)max_new) + 8) {
    qot_session_event_t ev;
    rc = qot_session_step(&s, &ev);
    ++steps;
    if (ev.kind == QOT_SESSION_EVENT_TOKEN)
      printf("token %u score %lld position %u\n", ev.result.token_id, (long long)ev.result.score_q26, ev.input_position);
    if (rc < 0) {
      printf("error %d\n", rc);
      break;
    }
  }
  printf("state %s stop %s\n", qot_session_state_name(s.state), qot_session_stop_reason_name(s.stop_reason));
  q4gpu_model_destroy(gpu);
  free(prompt);
  return rc < 0 ? 5 : 0;
}
