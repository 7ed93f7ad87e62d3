// json_config.cpp -- tcnn-style JSON configuration of a trainer.
//
// Mirrors try_create_from_config (include/tiny-metal-nn/factory_json.h:284-361)
// and the canonicalisation in include/tiny-metal-nn/detail/
// factory_json_detail.h:159-620: the same keys, defaults, aliases and
// validation rules, with errors reported as "path: message; ..." like
// format_error_diagnostics.  A small recursive-descent parser is included so
// the library has no JSON dependency.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/tmnn_cuda.h"
#include "runtime.h"

namespace tmnn {
namespace {

struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  bool is_int = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal *get(const std::string &k) const {
    for (auto &kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char *p;
  const char *end;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r')) ++p;
  }
  [[noreturn]] void fail(const char *what) {
    throw std::invalid_argument(std::string("json: ") + what);
  }
  JVal value() {
    ws();
    if (p >= end) fail("unexpected end");
    JVal v;
    if (*p == '{') {
      ++p;
      v.kind = JVal::Obj;
      ws();
      if (p < end && *p == '}') { ++p; return v; }
      for (;;) {
        ws();
        if (p >= end || *p != '"') fail("expected key");
        std::string k = string();
        ws();
        if (p >= end || *p != ':') fail("expected ':'");
        ++p;
        v.obj.emplace_back(k, value());
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; return v; }
        fail("expected ',' or '}'");
      }
    }
    if (*p == '[') {
      ++p;
      v.kind = JVal::Arr;
      ws();
      if (p < end && *p == ']') { ++p; return v; }
      for (;;) {
        v.arr.push_back(value());
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; return v; }
        fail("expected ',' or ']'");
      }
    }
    if (*p == '"') {
      v.kind = JVal::Str;
      v.str = string();
      return v;
    }
    if (!strncmp(p, "true", 4)) { p += 4; v.kind = JVal::Bool; v.b = true; return v; }
    if (!strncmp(p, "false", 5)) { p += 5; v.kind = JVal::Bool; return v; }
    if (!strncmp(p, "null", 4)) { p += 4; return v; }
    char *e = nullptr;
    v.num = strtod(p, &e);
    if (e == p) fail("bad value");
    v.is_int = true;
    for (const char *q = p; q < e; ++q)
      if (*q == '.' || *q == 'e' || *q == 'E') v.is_int = false;
    p = e;
    v.kind = JVal::Num;
    return v;
  }
  std::string string() {
    ++p;
    std::string s;
    while (p < end && *p != '"') {
      if (*p == '\\' && p + 1 < end) {
        ++p;
        switch (*p) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          default: s += *p;
        }
      } else {
        s += *p;
      }
      ++p;
    }
    if (p >= end) fail("unterminated string");
    ++p;
    return s;
  }
};

struct Diags {
  std::vector<std::string> errors;
  void err(const std::string &path, const std::string &msg) {
    errors.push_back(path + ": " + msg);
  }
};

void known_keys(const JVal &o, std::initializer_list<const char *> keys,
                const std::string &surface, Diags &d) {
  for (auto &kv : o.obj) {
    bool ok = false;
    for (auto *k : keys) ok |= kv.first == k;
    if (!ok) d.err(surface + "." + kv.first, "unknown key");
  }
}

double num(const JVal &o, const char *k, double def, const std::string &path,
           Diags &d) {
  const JVal *v = o.get(k);
  if (!v) return def;
  if (v->kind != JVal::Num) {
    d.err(path, "must be a number");
    return def;
  }
  return v->num;
}
int integer(const JVal &o, const char *k, int def, const std::string &path,
            Diags &d) {
  const JVal *v = o.get(k);
  if (!v) return def;
  if (v->kind != JVal::Num || !v->is_int) {
    d.err(path, "must be an integer");
    return def;
  }
  return (int)v->num;
}
std::string str(const JVal &o, const char *k, const char *def,
                const std::string &path, Diags &d) {
  const JVal *v = o.get(k);
  if (!v) return def;
  if (v->kind != JVal::Str) {
    d.err(path, "must be a string");
    return def;
  }
  return v->str;
}
bool boolean(const JVal &o, const char *k, bool def, const std::string &path,
             Diags &d) {
  const JVal *v = o.get(k);
  if (!v) return def;
  if (v->kind != JVal::Bool) {
    d.err(path, "must be a boolean");
    return def;
  }
  return v->b;
}
void positive(double v, const std::string &path, Diags &d) {
  if (!(v > 0)) d.err(path, "must be positive");
}

}  // namespace

// Parses and canonicalises a configuration; throws std::invalid_argument
// with the joined diagnostics on error.
void config_from_json(uint32_t n_input, uint32_t n_output, const char *text,
                      tmnn_spec *spec, tmnn_train_cfg *cfg) {
  if (!text) throw std::invalid_argument("create_from_config: null config");
  Parser ps{text, text + strlen(text)};
  JVal root = ps.value();
  ps.ws();
  if (ps.p != ps.end) throw std::invalid_argument("json: trailing characters");
  if (root.kind != JVal::Obj)
    throw std::invalid_argument("create_from_config: config must be an object");
  Diags d;
  known_keys(root, {"encoding", "network", "loss", "optimizer", "weight_init",
                    "batch_size", "training", "b200"},
             "config", d);
  static const JVal empty{JVal::Obj};
  auto section = [&](const char *k) -> const JVal & {
    const JVal *v = root.get(k);
    if (!v) return empty;
    if (v->kind != JVal::Obj) {
      d.err(k, "must be an object");
      return empty;
    }
    return *v;
  };
  tmnn_cuda_default_train_cfg(cfg);
  std::memset(spec, 0, sizeof *spec);

  // encoding (factory_json_detail.h:159-220)
  const JVal &enc = section("encoding");
  known_keys(enc, {"otype", "n_levels", "n_features_per_level",
                   "log2_hashmap_size", "base_resolution", "per_level_scale",
                   "interpolation"},
             "encoding", d);
  if (n_input == 0) d.err("encoding.n_input_dims", "must be >= 1");
  std::string eo = str(enc, "otype", "HashGrid", "encoding.otype", d);
  if (eo == "MultiresolutionHashGrid") eo = "HashGrid";
  if (eo != "HashGrid")
    d.err("encoding.otype", "unsupported encoding otype '" + eo + "'");
  spec->n_levels = integer(enc, "n_levels", 16, "encoding.n_levels", d);
  spec->n_features_per_level =
      integer(enc, "n_features_per_level", 2, "encoding.n_features_per_level", d);
  spec->log2_hashmap_size =
      integer(enc, "log2_hashmap_size", 19, "encoding.log2_hashmap_size", d);
  spec->base_resolution =
      (float)num(enc, "base_resolution", 16.0, "encoding.base_resolution", d);
  spec->per_level_scale =
      (float)num(enc, "per_level_scale", 1.447, "encoding.per_level_scale", d);
  positive(spec->n_levels, "encoding.n_levels", d);
  positive(spec->n_features_per_level, "encoding.n_features_per_level", d);
  positive(spec->log2_hashmap_size, "encoding.log2_hashmap_size", d);
  positive(spec->base_resolution, "encoding.base_resolution", d);
  positive(spec->per_level_scale, "encoding.per_level_scale", d);
  if (str(enc, "interpolation", "Linear", "encoding.interpolation", d) !=
      "Linear")
    d.err("encoding.interpolation",
          "only 'Linear' interpolation is supported by the current core "
          "descriptor bridge");
  spec->spatial_dims = (int32_t)n_input;

  // network (factory_json_detail.h:222-290)
  const JVal &net = section("network");
  known_keys(net, {"otype", "n_neurons", "n_hidden_layers", "activation",
                   "output_activation", "training"},
             "network", d);
  if (n_output == 0) d.err("network.n_output_dims", "must be >= 1");
  const std::string no = str(net, "otype", "FullyFusedMLP", "network.otype", d);
  if (no == "TiledMLP")
    d.err("network.otype", "TiledMLP JSON canonicalization is reserved for later C4");
  else if (no != "FullyFusedMLP")
    d.err("network.otype", "unsupported network otype '" + no + "'");
  spec->hidden_dim = integer(net, "n_neurons", 64, "network.n_neurons", d);
  spec->num_hidden_layers =
      integer(net, "n_hidden_layers", 2, "network.n_hidden_layers", d);
  positive(spec->hidden_dim, "network.n_neurons", d);
  positive(spec->num_hidden_layers, "network.n_hidden_layers", d);
  if (str(net, "activation", "ReLU", "network.activation", d) != "ReLU")
    d.err("network.activation",
          "only 'ReLU' activation is supported by the current FullyFusedMLP "
          "descriptor bridge");
  const std::string oa =
      str(net, "output_activation", "None", "network.output_activation", d);
  if (oa != "None" && oa != "Linear")
    d.err("network.output_activation",
          "only 'None' output activation is supported by the current "
          "FullyFusedMLP descriptor bridge");
  spec->num_outputs = (int32_t)n_output;

  // loss (factory_json_detail.h:403-440)
  const JVal *lj = root.get("loss");
  JVal loss_default{JVal::Obj};
  const JVal &loss = lj && lj->kind == JVal::Obj ? *lj : loss_default;
  if (lj && lj->kind != JVal::Obj) d.err("loss", "must be an object");
  const std::string lo = str(loss, "otype", "L2", "loss.otype", d);
  spec->huber_delta = 1.0f;
  if (lo == "L2") {
    known_keys(loss, {"otype"}, "loss", d);
    spec->loss = TMNN_LOSS_L2;
  } else if (lo == "L1") {
    known_keys(loss, {"otype"}, "loss", d);
    spec->loss = TMNN_LOSS_L1;
  } else if (lo == "Huber") {
    known_keys(loss, {"otype", "huber_delta"}, "loss", d);
    spec->loss = TMNN_LOSS_HUBER;
    spec->huber_delta = (float)num(loss, "huber_delta", 1.0, "loss.huber_delta", d);
    positive(spec->huber_delta, "loss.huber_delta", d);
  } else if (lo == "Cosine") {
    known_keys(loss, {"otype", "output_dims"}, "loss", d);
    spec->loss = TMNN_LOSS_COSINE;
    if (loss.get("output_dims") &&
        integer(loss, "output_dims", 0, "loss.output_dims", d) < 2)
      d.err("loss.output_dims", "must be >= 2 when provided");
  } else {
    d.err("loss.otype", "unsupported loss otype '" + lo + "'");
  }

  // optimizer (factory_json_detail.h:452-500); learning_rate feeds both
  // lr_encoding and lr_network (:467-468)
  const JVal &opt = section("optimizer");
  known_keys(opt, {"otype", "learning_rate", "beta1", "beta2", "epsilon",
                   "l1_reg", "l2_reg"},
             "optimizer", d);
  const std::string oo = str(opt, "otype", "Adam", "optimizer.otype", d);
  if (oo != "Adam")
    d.err("optimizer.otype", "unsupported optimizer otype '" + oo + "'");
  if (root.get("optimizer")) {
    const float lr =
        (float)num(opt, "learning_rate", 1e-3, "optimizer.learning_rate", d);
    positive(lr, "optimizer.learning_rate", d);
    if (opt.get("learning_rate")) cfg->lr_encoding = cfg->lr_network = lr;
    cfg->beta1 = (float)num(opt, "beta1", 0.9, "optimizer.beta1", d);
    cfg->beta2 = (float)num(opt, "beta2", 0.99, "optimizer.beta2", d);
    cfg->epsilon = (float)num(opt, "epsilon", 1e-15, "optimizer.epsilon", d);
    cfg->l1_reg = (float)num(opt, "l1_reg", 0.0, "optimizer.l1_reg", d);
    cfg->l2_reg = (float)num(opt, "l2_reg", 0.0, "optimizer.l2_reg", d);
    positive(cfg->beta1, "optimizer.beta1", d);
    positive(cfg->beta2, "optimizer.beta2", d);
    positive(cfg->epsilon, "optimizer.epsilon", d);
    if (cfg->l1_reg < 0) d.err("optimizer.l1_reg", "must be >= 0");
    if (cfg->l2_reg < 0) d.err("optimizer.l2_reg", "must be >= 0");
  }

  // weight_init (factory_json_detail.h:541-620)
  const JVal &wi = section("weight_init");
  known_keys(wi, {"hash_grid_init", "hash_grid_range", "mlp_init",
                  "mlp_nonlinearity", "mlp_uniform_range", "mlp_normal_stddev",
                  "mlp_kaiming_a", "seed"},
             "weight_init", d);
  const std::string hgi =
      str(wi, "hash_grid_init", "Uniform", "weight_init.hash_grid_init", d);
  if (hgi != "Uniform" && hgi != "Zero")
    d.err("weight_init.hash_grid_init",
          "unsupported value '" + hgi + "'; allowed: Uniform, Zero");
  cfg->hash_init = hgi == "Zero" ? 1 : 0;
  cfg->hash_init_range =
      (float)num(wi, "hash_grid_range", 1e-4, "weight_init.hash_grid_range", d);
  positive(cfg->hash_init_range, "weight_init.hash_grid_range", d);
  static const char *kMlp[] = {"KaimingUniform", "KaimingNormal",
                               "XavierUniform", "XavierNormal", "Uniform",
                               "Normal", "Zero"};
  const std::string mi =
      str(wi, "mlp_init", "KaimingUniform", "weight_init.mlp_init", d);
  cfg->mlp_init = -1;
  for (int i = 0; i < 7; ++i)
    if (mi == kMlp[i]) cfg->mlp_init = i;
  if (cfg->mlp_init < 0) {
    d.err("weight_init.mlp_init",
          "unsupported value '" + mi +
              "'; allowed: KaimingUniform, KaimingNormal, XavierUniform, "
              "XavierNormal, Uniform, Normal, Zero");
    cfg->mlp_init = 0;
  }
  static const char *kNl[] = {"Linear", "ReLU", "LeakyReLU", "Tanh", "Sigmoid"};
  const std::string nl =
      str(wi, "mlp_nonlinearity", "ReLU", "weight_init.mlp_nonlinearity", d);
  cfg->mlp_nonlinearity = -1;
  for (int i = 0; i < 5; ++i)
    if (nl == kNl[i]) cfg->mlp_nonlinearity = i;
  if (cfg->mlp_nonlinearity < 0) {
    d.err("weight_init.mlp_nonlinearity",
          "unsupported value '" + nl +
              "'; allowed: Linear, ReLU, LeakyReLU, Tanh, Sigmoid");
    cfg->mlp_nonlinearity = 1;
  }
  cfg->mlp_uniform_range = (float)num(wi, "mlp_uniform_range", 1e-2,
                                      "weight_init.mlp_uniform_range", d);
  positive(cfg->mlp_uniform_range, "weight_init.mlp_uniform_range", d);
  cfg->mlp_normal_stddev = (float)num(wi, "mlp_normal_stddev", 1e-2,
                                      "weight_init.mlp_normal_stddev", d);
  positive(cfg->mlp_normal_stddev, "weight_init.mlp_normal_stddev", d);
  cfg->mlp_kaiming_a =
      (float)num(wi, "mlp_kaiming_a", 0.0, "weight_init.mlp_kaiming_a", d);
  if (cfg->mlp_kaiming_a < 0) d.err("weight_init.mlp_kaiming_a", "must be >= 0");
  cfg->seed = (uint64_t)num(wi, "seed", 42.0, "weight_init.seed", d);

  // top-level batch_size (factory_json.h:322-331)
  if (root.get("batch_size")) {
    cfg->batch_size = integer(root, "batch_size", cfg->batch_size, "batch_size", d);
    positive(cfg->batch_size, "batch_size", d);
  }

  // this build's execution knobs
  const JVal &b2 = section("b200");
  known_keys(b2, {"family", "hash_grad_format", "table_dtype", "morton_sort",
                  "sparse_hash_adam", "active_levels", "numerics_sampling_mode",
                  "numerics_sample_interval", "bad_step_recovery",
                  "morton_key_bits", "enable_probes"},
             "b200", d);
  const std::string fam = str(b2, "family", "Auto", "b200.family", d);
  if (fam == "Auto") cfg->family = TMNN_FAMILY_AUTO;
  else if (fam == "FullyFused") cfg->family = TMNN_FAMILY_FULLY_FUSED;
  else if (fam == "Tiled") cfg->family = TMNN_FAMILY_TILED;
  else if (fam == "SafeDebug") cfg->family = TMNN_FAMILY_SAFE_DEBUG;
  else d.err("b200.family", "unsupported value '" + fam +
                                "'; allowed: Auto, FullyFused, Tiled, SafeDebug");
  const std::string gf = str(b2, "hash_grad_format", "Fixed16",
                             "b200.hash_grad_format", d);
  if (gf == "Fixed16") cfg->hash_grad_format = TMNN_GRAD_FIXED16;
  else if (gf == "F32") cfg->hash_grad_format = TMNN_GRAD_F32;
  else if (gf == "F16") cfg->hash_grad_format = TMNN_GRAD_F16;
  else d.err("b200.hash_grad_format", "unsupported value '" + gf +
                                          "'; allowed: Fixed16, F32, F16");
  const std::string td = str(b2, "table_dtype", "F32", "b200.table_dtype", d);
  if (td == "F32") spec->table_dtype = TMNN_DTYPE_F32;
  else if (td == "F16") spec->table_dtype = TMNN_DTYPE_F16;
  else d.err("b200.table_dtype", "unsupported value '" + td + "'; allowed: F32, F16");
  cfg->morton_sort = boolean(b2, "morton_sort", true, "b200.morton_sort", d) ? 1 : 0;
  if (b2.get("sparse_hash_adam"))
    cfg->sparse_hash_adam =
        boolean(b2, "sparse_hash_adam", true, "b200.sparse_hash_adam", d) ? 1 : 0;
  cfg->active_levels = integer(b2, "active_levels", 0, "b200.active_levels", d);
  // TrainerConfig::enable_probes (include/tiny-metal-nn/trainer.h:51-54)
  cfg->enable_probes =
      boolean(b2, "enable_probes", false, "b200.enable_probes", d) ? 1 : 0;
  if (b2.get("morton_key_bits")) {
    const int kb = integer(b2, "morton_key_bits", 12, "b200.morton_key_bits", d);
    if (kb < 0 || kb > 32)
      d.err("b200.morton_key_bits", "must be in [0, 32]");
    cfg->morton_key_bits = kb;
  }
  // RuntimePolicyOverrides (include/tiny-metal-nn/runtime_policy.h:43-52):
  // the numerics guard knobs, with the enum names of the reference
  if (b2.get("numerics_sampling_mode")) {
    const std::string m = str(b2, "numerics_sampling_mode", "Sampled",
                              "b200.numerics_sampling_mode", d);
    if (m == "Sampled") cfg->numerics_sampling_mode = TMNN_NUMERICS_SAMPLED;
    else if (m == "Periodic") cfg->numerics_sampling_mode = TMNN_NUMERICS_PERIODIC;
    else if (m == "FullPerStep") cfg->numerics_sampling_mode = TMNN_NUMERICS_FULL;
    else if (m == "Disabled") cfg->numerics_sampling_mode = TMNN_NUMERICS_DISABLED;
    else d.err("b200.numerics_sampling_mode",
               "unsupported value '" + m +
                   "'; allowed: Sampled, Periodic, FullPerStep, Disabled");
  }
  if (b2.get("numerics_sample_interval")) {
    const int n = integer(b2, "numerics_sample_interval", 128,
                          "b200.numerics_sample_interval", d);
    cfg->numerics_sample_interval = n > 0 ? n : 1;
  }
  if (b2.get("bad_step_recovery")) {
    const std::string m = str(b2, "bad_step_recovery", "SignalOnly",
                              "b200.bad_step_recovery", d);
    if (m == "SignalOnly") cfg->bad_step_recovery = TMNN_BAD_STEP_SIGNAL_ONLY;
    else if (m == "Throw") cfg->bad_step_recovery = TMNN_BAD_STEP_THROW;
    else if (m == "Skip") cfg->bad_step_recovery = TMNN_BAD_STEP_SKIP;
    else if (m == "Rollback") cfg->bad_step_recovery = TMNN_BAD_STEP_ROLLBACK;
    else if (m == "FallbackAndRetryWithSafeFamily")
      cfg->bad_step_recovery = TMNN_BAD_STEP_SAFE_FAMILY_RETRY;
    else d.err("b200.bad_step_recovery",
               "unsupported value '" + m +
                   "'; allowed: SignalOnly, Throw, Skip, Rollback, "
                   "FallbackAndRetryWithSafeFamily");
  }

  if (!d.errors.empty()) {
    std::string msg = "create_from_config: ";
    for (size_t i = 0; i < d.errors.size(); ++i)
      msg += (i ? "; " : "") + d.errors[i];
    throw std::invalid_argument(msg);
  }
}

}  // namespace tmnn
