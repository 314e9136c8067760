// pz_params.cpp — sampler settings from the front ends of the generate loop:
// command-line flags (the reference's src/cli/args.c) and the JSON body of
// an OpenAI-style chat-completions request (its src/api/json_parse.c, with
// the clamps of src/api/http_server.c:413-418).  Host code only.
//
// The reference parses only temperature and top_p (and a --seed it never
// uses: args.c:125-126 against generate.c:126).  These parsers take the same
// flags and fields with the same defaults and clamps, plus the settings the
// batch sampler adds (top-k, the three penalties, the seed, logprobs), and
// fill a pz_sampling_params ready for pz_sample_batch and pz_rng_seed_batch.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "../../include/pz_sampling.h"

namespace {

pz_sampling_params defaults(float temperature, float top_p) {
  pz_sampling_params p;
  std::memset(&p, 0, sizeof p);
  p.cfg.temperature = temperature;
  p.cfg.top_k = 0;
  p.cfg.top_p = top_p;
  p.cfg.repetition_penalty = 1.0f;
  p.cfg.frequency_penalty = 0.0f;
  p.cfg.presence_penalty = 0.0f;
  p.seed = -1;
  p.logprobs = 0;
  p.top_logprobs = 0;
  return p;
}

// ---- a minimal JSON reader: enough to walk one object's top-level keys ----
struct Reader {
  const char *p;
  void ws() {
    while (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r') p++;
  }
  bool lit(const char *s) {
    const size_t n = std::strlen(s);
    if (std::strncmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  // A string into out (escapes kept verbatim except \" and \\; keys are plain).
  bool str(char *out, size_t cap) {
    ws();
    if (*p != '"') return false;
    p++;
    size_t n = 0;
    while (*p && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (!*p) return false;
        c = *p++;
        if (c == 'u') {  // \uXXXX: skip the four hex digits
          for (int i = 0; i < 4; i++)
            if (!*p++) return false;
          c = '?';
        }
      }
      if (out && n + 1 < cap) out[n++] = c;
    }
    if (*p != '"') return false;
    p++;
    if (out && cap) out[n] = '\0';
    return true;
  }
  bool number(double *v) {
    ws();
    char *end = nullptr;
    const double d = std::strtod(p, &end);
    if (end == p) return false;
    p = end;
    *v = d;
    return true;
  }
  // true/false (1/0) or null (-1); -2 when neither
  int boolean() {
    ws();
    if (lit("true")) return 1;
    if (lit("false")) return 0;
    if (lit("null")) return -1;
    return -2;
  }
  // Skips any value (nested objects and arrays included).
  bool skip() {
    ws();
    if (*p == '"') return str(nullptr, 0);
    if (*p == '{' || *p == '[') {
      int depth = 0;
      do {
        if (*p == '"') {
          if (!str(nullptr, 0)) return false;
          continue;
        }
        if (*p == '{' || *p == '[') depth++;
        if (*p == '}' || *p == ']') depth--;
        if (!*p) return false;
        p++;
      } while (depth > 0);
      return true;
    }
    if (boolean() >= -1) return true;
    double d;
    return number(&d);
  }
};

}  // namespace

extern "C" {

void pz_params_init_cli(pz_sampling_params *p) {
  if (p) *p = defaults(0.7f, 0.9f);  // reference src/cli/args.c:82-83, seed -1 at :89
}

void pz_params_init_api(pz_sampling_params *p) {
  if (p) *p = defaults(1.0f, 1.0f);  // reference src/api/json_parse.c:299-300
}

pz_status pz_params_from_args(pz_sampling_params *p, int argc, char **argv) {
  if (!p || argc < 0 || (argc > 0 && !argv)) return PZ_ERR_INVALID_ARGS;
  pz_params_init_cli(p);
  for (int i = 1; i < argc; i++) {
    const char *a = argv[i];
    if (!a) continue;
    const bool has = i + 1 < argc && argv[i + 1];
    // the reference's flags (args.c:117-120, :125-126), atof/atoi as there
    if (!std::strcmp(a, "--temperature") && has) {
      p->cfg.temperature = static_cast<float>(std::atof(argv[++i]));
    } else if (!std::strcmp(a, "--top-p") && has) {
      p->cfg.top_p = static_cast<float>(std::atof(argv[++i]));
    } else if (!std::strcmp(a, "--seed") && has) {
      p->seed = std::atoi(argv[++i]);
    // the batch sampler's additions
    } else if (!std::strcmp(a, "--top-k") && has) {
      p->cfg.top_k = std::atoi(argv[++i]);
    } else if (!std::strcmp(a, "--repeat-penalty") && has) {
      p->cfg.repetition_penalty = static_cast<float>(std::atof(argv[++i]));
    } else if (!std::strcmp(a, "--frequency-penalty") && has) {
      p->cfg.frequency_penalty = static_cast<float>(std::atof(argv[++i]));
    } else if (!std::strcmp(a, "--presence-penalty") && has) {
      p->cfg.presence_penalty = static_cast<float>(std::atof(argv[++i]));
    } else if (!std::strcmp(a, "--logprobs")) {
      p->logprobs = 1;
    } else if (!std::strcmp(a, "--top-logprobs") && has) {
      p->logprobs = 1;
      p->top_logprobs = std::atoi(argv[++i]);
    }
    // anything else belongs to the caller's own parser
  }
  if (p->top_logprobs < 0) p->top_logprobs = 0;
  if (p->top_logprobs > PZ_TOP_LOGPROBS_MAX) p->top_logprobs = PZ_TOP_LOGPROBS_MAX;
  return PZ_OK;
}

pz_status pz_params_from_json(pz_sampling_params *p, const char *json) {
  if (!p || !json) return PZ_ERR_INVALID_ARGS;
  pz_params_init_api(p);
  Reader r{json};
  r.ws();
  if (*r.p != '{') return PZ_ERR_INVALID_ARGS;
  r.p++;
  for (;;) {
    r.ws();
    if (*r.p == '}') break;
    char key[64];
    if (!r.str(key, sizeof key)) return PZ_ERR_INVALID_ARGS;
    r.ws();
    if (*r.p != ':') return PZ_ERR_INVALID_ARGS;
    r.p++;
    double v = 0.0;
    int b = -2;
    bool ok = true;
    if (!std::strcmp(key, "temperature")) {
      ok = r.number(&v) && ((p->cfg.temperature = static_cast<float>(v)), true);
    } else if (!std::strcmp(key, "top_p")) {
      ok = r.number(&v) && ((p->cfg.top_p = static_cast<float>(v)), true);
    } else if (!std::strcmp(key, "top_k")) {
      ok = r.number(&v) && ((p->cfg.top_k = static_cast<int32_t>(v)), true);
    } else if (!std::strcmp(key, "repetition_penalty")) {
      ok = r.number(&v) && ((p->cfg.repetition_penalty = static_cast<float>(v)), true);
    } else if (!std::strcmp(key, "frequency_penalty")) {
      ok = r.number(&v) && ((p->cfg.frequency_penalty = static_cast<float>(v)), true);
    } else if (!std::strcmp(key, "presence_penalty")) {
      ok = r.number(&v) && ((p->cfg.presence_penalty = static_cast<float>(v)), true);
    } else if (!std::strcmp(key, "seed")) {
      r.ws();
      if (r.lit("null")) {
        p->seed = -1;
      } else {
        ok = r.number(&v) && ((p->seed = static_cast<int64_t>(v)), true);
      }
    } else if (!std::strcmp(key, "logprobs")) {
      b = r.boolean();
      ok = b >= -1;
      p->logprobs = b == 1 ? 1 : 0;
    } else if (!std::strcmp(key, "top_logprobs")) {
      r.ws();
      if (!r.lit("null")) ok = r.number(&v) && ((p->top_logprobs = static_cast<int32_t>(v)), true);
    } else {
      ok = r.skip();
    }
    if (!ok) return PZ_ERR_INVALID_ARGS;
    r.ws();
    if (*r.p == ',') {
      r.p++;
      continue;
    }
    if (*r.p != '}') return PZ_ERR_INVALID_ARGS;
  }
  // the API's clamps (reference src/api/http_server.c:415-417) ...
  float &t = p->cfg.temperature;
  if (t < 0.0f) t = 0.0f;
  if (t > 2.0f) t = 2.0f;
  float &tp = p->cfg.top_p;
  if (tp < 0.0f || tp > 1.0f) tp = 1.0f;
  // ... and the OpenAI ranges of the added fields
  p->cfg.frequency_penalty = std::fmax(-2.0f, std::fmin(2.0f, p->cfg.frequency_penalty));
  p->cfg.presence_penalty = std::fmax(-2.0f, std::fmin(2.0f, p->cfg.presence_penalty));
  if (!(p->cfg.repetition_penalty > 0.0f)) p->cfg.repetition_penalty = 1.0f;
  if (p->cfg.top_k < 0) p->cfg.top_k = 0;
  if (p->top_logprobs < 0) p->top_logprobs = 0;
  if (p->top_logprobs > PZ_TOP_LOGPROBS_MAX) p->top_logprobs = PZ_TOP_LOGPROBS_MAX;
  if (p->top_logprobs > 0) p->logprobs = 1;
  return PZ_OK;
}

}  // extern "C"
