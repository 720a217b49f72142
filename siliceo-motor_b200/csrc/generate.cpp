// Autoregressive loop over any device (crates/s-models/src/generate.rs:149-250).
//
// The device fuses forward_cached and sampling (only the token id leaves the
// GPU), so a step's masker runs before that step's forward instead of after
// it; on_prefill still runs once, right after the prefill forward, with the
// cache holding exactly the prompt.
#include <chrono>
#include <string>
#include <vector>

#include "../../include/sm_engine.h"
#include "common.hpp"

using namespace sm;

extern "C" {

int sm_generate_with(const sm_device_vtbl* vt, void* dev, uint64_t vocab, const uint32_t* prompt, uint64_t n_prompt,
                     const sm_gen_params* p, const uint32_t* eos, uint64_t n_eos, sm_on_token_fn on_token,
                     sm_masker_fn masker, sm_stop_fn stop, sm_on_prefill_fn on_prefill, void* ud, void* seed_cache,
                     uint64_t seed_n, uint32_t* out_ids, sm_gen_result* res) {
  if (!vt || !vt->new_cache || !vt->free_cache || !vt->forward_sample || !p || !res || (p->max_tokens && !out_ids)) {
    set_error("sm_generate: bad arguments");
    return SM_ERR_ARG;
  }
  if (n_prompt == 0 || !prompt) {
    set_error("sm_generate: empty prompt");
    return SM_ERR_ARG;
  }
  const auto t0 = std::chrono::steady_clock::now();
  const sm_sampler smp{p->temperature, p->top_k, p->top_p};
  const uint64_t seed = p->has_seed ? p->seed
                                    : (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                          std::chrono::system_clock::now().time_since_epoch())
                                          .count();
  uint64_t rng = sm_rng_seed(seed);  // Rng::new (sampling.rs:15-17)
  const uint64_t max_seq = n_prompt + p->max_tokens;
  // usable seed: a strict, non-empty prefix of the prompt (generate.rs:185-188)
  const bool usable = seed_cache && seed_n > 0 && seed_n < n_prompt;
  void* cache = nullptr;
  int rc;
  if (usable) {
    cache = seed_cache;
  } else if ((rc = vt->new_cache(dev, max_seq, &cache)) != SM_OK) {
    return rc;
  }
  const uint32_t* in = usable ? prompt + seed_n : prompt;
  const uint64_t n_in = usable ? n_prompt - seed_n : n_prompt;
  std::vector<uint8_t> mask(vocab ? vocab : 1);
  uint64_t n = 0;
  int32_t finish_stop = 0;
  uint32_t last = prompt[n_prompt - 1];
  rc = SM_OK;
  if (p->max_tokens == 0) {  // prefill only: the state is still produced for on_prefill
    const sm_sampler greedy{0.f, -1, -1.f};
    uint64_t r2 = rng;
    uint32_t tok;
    rc = vt->forward_sample(dev, cache, in, n_in, &greedy, &r2, nullptr, &tok);
    if (rc == SM_OK && on_prefill) on_prefill(ud, cache);
  }
  for (uint64_t step = 0; step < p->max_tokens && rc == SM_OK; step++) {
    const bool has_mask = masker && vocab && masker(ud, mask.data(), vocab);
    uint32_t next = 0;
    if (step == 0) {
      rc = vt->forward_sample(dev, cache, in, n_in, &smp, &rng, has_mask ? mask.data() : nullptr, &next);
      if (rc != SM_OK) break;
      if (on_prefill) on_prefill(ud, cache);
    } else {
      rc = vt->forward_sample(dev, cache, &last, 1, &smp, &rng, has_mask ? mask.data() : nullptr, &next);
      if (rc != SM_OK) break;
    }
    out_ids[n++] = next;
    last = next;
    if (on_token && !on_token(ud, next)) { finish_stop = 1; break; }  // consumer abort
    bool is_eos = false;
    for (uint64_t i = 0; i < n_eos; i++) is_eos |= eos[i] == next;
    if (is_eos) { finish_stop = 1; break; }
    if (stop && stop(ud, out_ids, n)) { finish_stop = 1; break; }
  }
  if (!usable) {
    std::string err = rc == SM_OK ? std::string() : get_error();
    vt->free_cache(dev, cache);
    if (rc != SM_OK) set_error(err);
  }
  if (rc != SM_OK) return rc;
  res->n_ids = n;
  res->finish_stop = finish_stop;
  res->prompt_tokens = n_prompt;
  res->prefix_reused = usable ? seed_n : 0;
  res->elapsed_secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return SM_OK;
}

static int eng_new_cache(void* dev, uint64_t max_seq, void** cache) {
  return sm_cache_new((sm_model*)dev, max_seq, (sm_cache**)cache);
}
static int eng_free_cache(void*, void* cache) { return sm_cache_free((sm_cache*)cache); }
static int eng_forward_sample(void* dev, void* cache, const uint32_t* t, uint64_t n, const sm_sampler* s, uint64_t* rng,
                              const uint8_t* mask, uint32_t* out) {
  return sm_forward_sample((sm_model*)dev, (sm_cache*)cache, t, n, s, rng, mask, out);
}

int sm_generate(sm_model* m, const uint32_t* prompt, uint64_t n_prompt, const sm_gen_params* params, const uint32_t* eos,
                uint64_t n_eos, sm_on_token_fn on_token, sm_masker_fn masker, sm_stop_fn stop,
                sm_on_prefill_fn on_prefill, void* ud, sm_cache* seed_cache, uint64_t seed_n, uint32_t* out_ids,
                sm_gen_result* res) {
  sm_config c;
  if (sm_model_config(m, &c) != SM_OK) return SM_ERR_ARG;
  if (seed_cache) {
    uint64_t len = 0;
    sm_cache_len(seed_cache, &len);
    if (seed_n > 0 && seed_n < n_prompt && len != seed_n) {
      set_error("sm_generate: the seed cache length must equal seed_n");
      return SM_ERR_STATE;
    }
  }
  static const sm_device_vtbl vt{eng_new_cache, eng_free_cache, eng_forward_sample};
  return sm_generate_with(&vt, m, c.vocab_size, prompt, n_prompt, params, eos, n_eos, on_token, masker, stop, on_prefill,
                          ud, seed_cache, seed_n, out_ids, res);
}

}  // extern "C"
