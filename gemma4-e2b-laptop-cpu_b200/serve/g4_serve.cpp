// g4_serve: the reference engine's process interface (gemma4_engine.cpp:1681-1689, read by
// server/server.py:44-75) over the library's request API, so the reference's server can start this
// binary in place of its engine.
//
//   g4_serve <ckpt> <index> <prompt file> <n_new>
//
// When <ckpt> exists (a checkpoint directory holding model.safetensors, or the file itself), the
// target weights are loaded from it (g4_engine_create_from_checkpoint), through <index> when that
// file exists (the reference's make_index.py output) and the safetensors header otherwise; else the
// model is the synthetic one, generated from a seed on the device.  With ENGINE_SERVE set, each stdin line is a request "<n_new> <id> <id> ..."
// or "BENCH_MODE <k> <tree>"; otherwise one request runs with the token ids of <prompt file>
// (whitespace separated) and <n_new>.  Per request the output is, as the reference prints it:
//   FIRST <id>                       (n_new > 0: the token after the prompt, before decoding)
//   TOK <id> ...                     (ENGINE_STREAM set: each round's committed tokens)
//   GEN: <id> ...
//   TIMING prompt=.. reused=.. new=.. prefill_s=.. decode_tokens=.. decode_s=.. decode_tok_s=..
//          tokens_per_round=.. ngram_rounds=a/b ngram_acc_per_round=.. slot=..
// Engine settings come from the reference's variables where this build has them: ENGINE_K,
// ENGINE_NGRAM, ENGINE_NGLEN, ENGINE_PREFILL_INT8, ENGINE_DECODE_INT8, ENGINE_HEAD_SCREEN,
// ENGINE_CTX, ENGINE_FAKE_CTX, ENGINE_ATT_PAR, ENGINE_PREFILL_BLOCK, ENGINE_SLOTS,
// ENGINE_SLOT_MIN_REUSE, ENGINE_STREAM; the synthetic model's size from G4_HIDDEN, G4_LAYERS, G4_MLP,
// G4_VOCAB, G4_SEED, G4_KV_OWNERS (defaults: configs[4], no KV sharing).  Not built here: the audio tower (AUDIO_* lines answer
// "AUDIO_UNSUPPORTED"; "A=" words of a request are skipped) and the tree/sibling mode (BENCH_MODE
// with tree 1 answers MODE_ERROR).
#include <sys/stat.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "g4.h"

namespace {

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v ? std::atoi(v) : dflt;
}

bool is_stop(int t) { return t == 106 || t == 1; }

// Streaming state of one request (the reference's emit, :1611-1613).
struct Emit {
  std::vector<int> gen;
  size_t emitted = 1;
  int n_new = 0;
  bool stream = false;
};

void on_tokens(const int32_t* toks, int n, void* user) {
  Emit& s = *static_cast<Emit*>(user);
  const bool first = s.gen.empty();
  for (int i = 0; i < n; ++i) s.gen.push_back(toks[i]);
  if (first) {
    std::printf("FIRST %d\n", s.gen[0]);
    std::fflush(stdout);
    return;
  }
  if (!s.stream) return;
  const size_t lim = std::min(s.gen.size(), (size_t)s.n_new);
  std::string o;
  size_t i = s.emitted;
  for (; i < lim; ++i) {
    o += ' ';
    o += std::to_string(s.gen[i]);
    if (is_stop(s.gen[i])) { ++i; break; }
  }
  if (i > s.emitted) {
    std::printf("TOK%s\n", o.c_str());
    std::fflush(stdout);
    s.emitted = is_stop(s.gen[i - 1]) ? lim : i;
  }
}

int run_request(g4_engine* e, const std::vector<int>& prompt, int n_new, bool stream) {
  g4_request_info info{};
  int n_out = 0;
  std::vector<int32_t> out((size_t)std::max(1, n_new));
  Emit em;
  em.n_new = n_new;
  em.stream = stream;
  const int rc = g4_engine_request(e, prompt.data(), (int)prompt.size(), std::max(0, n_new), out.data(), &n_out, &info,
                                   n_new > 0 ? on_tokens : nullptr, &em);
  if (rc != G4_OK) {
    std::fprintf(stderr, "g4_serve: request failed: %s\n", g4_last_error());
    return rc;
  }
  const int n = (int)prompt.size();
  if (n_new <= 0) {
    std::printf("GEN:\nTIMING prompt=%d reused=%d new=%d prefill_s=%.3f decode_tokens=0 decode_s=0 decode_tok_s=0 "
                "tokens_per_round=0 ngram_rounds=0/0 ngram_acc_per_round=0\n",
                n, info.reused, n - info.reused, info.prefill_ms / 1e3);
    std::fflush(stdout);
    return G4_OK;
  }
  std::printf("GEN:");
  for (int i = 0; i < n_out; ++i) std::printf(" %d", out[i]);
  std::printf("\n");
  const int produced = std::max(0, n_out - 1);
  const double td = info.decode_ms / 1e3;
  std::printf("TIMING prompt=%d reused=%d new=%d prefill_s=%.3f decode_tokens=%d decode_s=%.3f decode_tok_s=%.2f "
              "tokens_per_round=%.2f ngram_rounds=%d/%d ngram_acc_per_round=%.2f slot=%d\n",
              n, info.reused, n - info.reused, info.prefill_ms / 1e3, produced, td, td > 0 ? produced / td : 0.0,
              info.rounds ? (double)produced / info.rounds : 1.0, info.ngram_rounds, info.rounds,
              info.ngram_rounds ? (double)info.ngram_accepted / info.ngram_rounds : 0.0, info.slot);
  std::fflush(stdout);
  return G4_OK;
}

void usage() {
  std::fprintf(stderr,
               "usage: g4_serve <ckpt> <index> <prompt file> <n_new>\n"
               "  ENGINE_SERVE=1: requests \"<n_new> <id> ...\" and \"BENCH_MODE <k> <tree>\" on stdin\n");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc >= 2 && (!std::strcmp(argv[1], "--help") || !std::strcmp(argv[1], "-h"))) {
    usage();
    return 0;
  }
  if (argc < 5) {
    usage();
    return 2;
  }
  g4_engine_config c;
  g4_engine_default_config(&c);
  c.hidden = env_int("G4_HIDDEN", c.hidden);
  c.n_layers = env_int("G4_LAYERS", c.n_layers);
  c.mlp = env_int("G4_MLP", c.mlp);
  c.vocab = env_int("G4_VOCAB", c.vocab);
  if (const char* s = std::getenv("G4_SEED")) c.seed = std::strtoull(s, nullptr, 10);
  c.kv_owners = env_int("G4_KV_OWNERS", c.kv_owners);
  c.ctx_max = env_int("ENGINE_CTX", c.ctx_max);
  c.k_draft = env_int("ENGINE_K", c.k_draft);
  c.ngram = env_int("ENGINE_NGRAM", c.ngram);
  c.ngram_len = std::min(7, env_int("ENGINE_NGLEN", c.ngram_len));
  c.prefill_int8 = env_int("ENGINE_PREFILL_INT8", c.prefill_int8) == 1 ? 1 : 0;
  c.decode_int8 = env_int("ENGINE_DECODE_INT8", c.decode_int8) == 0 ? 0 : 1;
  if (std::getenv("ENGINE_HEAD_SCREEN")) c.head_screen = env_int("ENGINE_HEAD_SCREEN", 1);
  c.att_par = env_int("ENGINE_ATT_PAR", c.att_par);
  c.prefill_block = env_int("ENGINE_PREFILL_BLOCK", c.prefill_block);
  c.slots = std::max(1, env_int("ENGINE_SLOTS", c.slots));
  c.slot_min_reuse = env_int("ENGINE_SLOT_MIN_REUSE", c.slot_min_reuse);
  if (c.k_draft == 0) c.ngram = 0;  // the reference's plain greedy loop when no drafts (:1614)
  g4_engine* e = nullptr;
  struct stat sb;
  const bool from_ckpt = stat(argv[1], &sb) == 0;
  if (from_ckpt) {
    g4_checkpoint* ck = nullptr;
    const bool has_index = stat(argv[2], &sb) == 0 && S_ISREG(sb.st_mode);
    if (g4_checkpoint_open(argv[1], has_index ? argv[2] : nullptr, &ck) != G4_OK ||
        g4_engine_create_from_checkpoint(&c, ck, &e) != G4_OK) {
      std::fprintf(stderr, "g4_serve: checkpoint %s: %s\n", argv[1], g4_last_error());
      g4_checkpoint_close(ck);
      return 1;
    }
    g4_checkpoint_config(ck, &c);
    g4_checkpoint_close(ck);
  } else if (g4_engine_create(&c, &e) != G4_OK) {
    std::fprintf(stderr, "g4_serve: engine: %s\n", g4_last_error());
    return 1;
  }
  if (const int fake = env_int("ENGINE_FAKE_CTX", 0); fake > 0 && g4_engine_fake_ctx(e, fake) != G4_OK) {
    std::fprintf(stderr, "g4_serve: fake context: %s\n", g4_last_error());
    return 1;
  }
  std::fprintf(stderr, "g4_serve: %s model hidden=%d layers=%d vocab=%d ctx=%d k=%d ngram=%d slots=%d\n", from_ckpt ? "checkpoint" : "synthetic",
               c.hidden, c.n_layers, c.vocab, c.ctx_max, c.k_draft, c.ngram, c.slots);
  const bool stream = std::getenv("ENGINE_STREAM") != nullptr;
  int rc = 0;
  if (std::getenv("ENGINE_SERVE")) {
    std::string line;
    while (std::getline(std::cin, line)) {
      if (line.rfind("BENCH_MODE ", 0) == 0) {
        std::stringstream ms(line);
        std::string cmd;
        int k = -1, tree = -1;
        ms >> cmd >> k >> tree;
        if (k >= 1 && k <= 3 && tree == 0 && c.drafter && g4_engine_set_k_draft(e, k) == G4_OK)
          std::printf("MODE k=%d tree=%d\n", k, tree);
        else
          std::printf("MODE_ERROR\n");
        std::fflush(stdout);
        continue;
      }
      if (line.rfind("AUDIO_", 0) == 0) {
        std::printf("AUDIO_UNSUPPORTED\n");
        std::fflush(stdout);
        continue;
      }
      std::stringstream ss(line);
      int n_new;
      if (!(ss >> n_new)) continue;
      std::vector<int> prompt;
      std::string w;
      while (ss >> w)
        if (w.rfind("A=", 0) != 0) prompt.push_back(std::atoi(w.c_str()));
      if (prompt.empty()) continue;
      if ((rc = run_request(e, prompt, n_new, stream)) != G4_OK) break;
    }
  } else {
    std::ifstream pf(argv[3]);
    std::vector<int> prompt;
    int t;
    while (pf >> t) prompt.push_back(t);
    if (prompt.empty()) {
      std::fprintf(stderr, "g4_serve: no token ids in %s\n", argv[3]);
      rc = 2;
    } else {
      rc = run_request(e, prompt, std::atoi(argv[4]), stream);
    }
  }
  g4_engine_destroy(e);
  return rc == G4_OK ? 0 : 1;
}
