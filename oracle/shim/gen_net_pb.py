#!/usr/bin/env python3
"""Generate a header-only stand-in for the protobuf classes of the MetalFish
weight format, so the reference's CPU backend compiles without protoc or
libprotobuf (neither is in this image).

TEST INFRASTRUCTURE ONLY: the header is used by the oracle build (the
reference's own ``Cpu::CpuNetwork`` compiled unmodified) and never by the
product library.

The message/field table below restates the schema of
``src/nn/proto/net.proto`` (package ``MetalFishNN``): the field names, numbers
and wire types must be identical so that (a) the reference sources compile
against the generated accessors, and (b) real ``.pb`` weight files decode.
The emitted C++ follows the accessor conventions of protobuf's generated code
(``x()``, ``has_x()``, ``set_x()``, ``mutable_x()``, ``add_x()``, ``x_size()``,
``clear_x()``) plus a small wire-format reader/writer.

Usage: python gen_net_pb.py <out_dir>   (writes out_dir/proto/net.pb.h and
out_dir/google/protobuf/io/{coded_stream,zero_copy_stream_impl}.h)
"""
import os
import sys

# ---------------------------------------------------------------- schema table
# kinds: u32 (varint), f32 (fixed32 float), fx32 (fixed32 int), bytes, str,
#        enum:<EnumName>, msg:<Type>; "rep" marks repeated fields.
ENUMS = {
    "Weights.Layer.Encoding": [("UNKNOWN_ENCODING", 0), ("LINEAR16", 1), ("FLOAT16", 2),
                               ("BFLOAT16", 3), ("FLOAT32", 4)],
    "NetworkFormat.InputFormat": [
        ("INPUT_UNKNOWN", 0), ("INPUT_CLASSICAL_112_PLANE", 1),
        ("INPUT_112_WITH_CASTLING_PLANE", 2), ("INPUT_112_WITH_CANONICALIZATION", 3),
        ("INPUT_112_WITH_CANONICALIZATION_HECTOPLIES", 4),
        ("INPUT_112_WITH_CANONICALIZATION_HECTOPLIES_ARMAGEDDON", 132),
        ("INPUT_112_WITH_CANONICALIZATION_V2", 5),
        ("INPUT_112_WITH_CANONICALIZATION_V2_ARMAGEDDON", 133)],
    "NetworkFormat.OutputFormat": [("OUTPUT_UNKNOWN", 0), ("OUTPUT_CLASSICAL", 1), ("OUTPUT_WDL", 2)],
    "NetworkFormat.NetworkStructure": [
        ("NETWORK_UNKNOWN", 0), ("NETWORK_CLASSICAL", 1), ("NETWORK_SE", 2),
        ("NETWORK_CLASSICAL_WITH_HEADFORMAT", 3), ("NETWORK_SE_WITH_HEADFORMAT", 4),
        ("NETWORK_ONNX", 5), ("NETWORK_ATTENTIONBODY_WITH_HEADFORMAT", 6),
        ("NETWORK_ATTENTIONBODY_WITH_MULTIHEADFORMAT", 7),
        ("NETWORK_AB_LEGACY_WITH_MULTIHEADFORMAT", 134)],
    "NetworkFormat.PolicyFormat": [("POLICY_UNKNOWN", 0), ("POLICY_CLASSICAL", 1),
                                   ("POLICY_CONVOLUTION", 2), ("POLICY_ATTENTION", 3)],
    "NetworkFormat.ValueFormat": [("VALUE_UNKNOWN", 0), ("VALUE_CLASSICAL", 1), ("VALUE_WDL", 2),
                                  ("VALUE_PARAM", 3)],
    "NetworkFormat.MovesLeftFormat": [("MOVES_LEFT_NONE", 0), ("MOVES_LEFT_V1", 1)],
    "NetworkFormat.ActivationFunction": [
        ("ACTIVATION_DEFAULT", 0), ("ACTIVATION_MISH", 1), ("ACTIVATION_RELU", 2),
        ("ACTIVATION_NONE", 3), ("ACTIVATION_TANH", 4), ("ACTIVATION_SIGMOID", 5),
        ("ACTIVATION_SELU", 6), ("ACTIVATION_SWISH", 7), ("ACTIVATION_RELU_2", 8),
        ("ACTIVATION_SOFTMAX", 9)],
    "NetworkFormat.DefaultActivation": [("DEFAULT_ACTIVATION_RELU", 0), ("DEFAULT_ACTIVATION_MISH", 1)],
    "NetworkFormat.InputEmbeddingFormat": [("INPUT_EMBEDDING_NONE", 0), ("INPUT_EMBEDDING_PE_MAP", 1),
                                           ("INPUT_EMBEDDING_PE_DENSE", 2)],
    "Format.Encoding": [("UNKNOWN", 0), ("LINEAR16", 1)],
    "OnnxModel.DataType": [("UNKNOWN_DATATYPE", 0), ("FLOAT", 1), ("FLOAT16", 10), ("BFLOAT16", 16)],
}

L = "msg:Weights.Layer"
CB = "msg:Weights.ConvBlock"
ENC = "msg:Weights.EncoderLayer"
# messages in dependency order (a message only refers to earlier ones)
MESSAGES = [
    ("EngineVersion", [("major", 1, "u32"), ("minor", 2, "u32"), ("patch", 3, "u32")]),
    ("Weights.Layer", [("min_val", 1, "f32"), ("max_val", 2, "f32"), ("params", 3, "bytes"),
                       ("encoding", 4, "enum:Weights.Layer.Encoding"), ("dims", 5, "u32", "rep")]),
    ("Weights.ConvBlock", [("weights", 1, L), ("biases", 2, L), ("bn_means", 3, L),
                           ("bn_stddivs", 4, L), ("bn_gammas", 5, L), ("bn_betas", 6, L)]),
    ("Weights.SEunit", [("w1", 1, L), ("b1", 2, L), ("w2", 3, L), ("b2", 4, L)]),
    ("Weights.Residual", [("conv1", 1, CB), ("conv2", 2, CB), ("se", 3, "msg:Weights.SEunit")]),
    ("Weights.Smolgen", [("compress", 1, L), ("dense1_w", 2, L), ("dense1_b", 3, L),
                         ("ln1_gammas", 4, L), ("ln1_betas", 5, L), ("dense2_w", 6, L),
                         ("dense2_b", 7, L), ("ln2_gammas", 8, L), ("ln2_betas", 9, L)]),
    ("Weights.MHA", [("q_w", 1, L), ("q_b", 2, L), ("k_w", 3, L), ("k_b", 4, L), ("v_w", 5, L),
                     ("v_b", 6, L), ("dense_w", 7, L), ("dense_b", 8, L),
                     ("smolgen", 9, "msg:Weights.Smolgen"), ("rpe_q", 10, L), ("rpe_k", 11, L),
                     ("rpe_v", 12, L)]),
    ("Weights.FFN", [("dense1_w", 1, L), ("dense1_b", 2, L), ("dense2_w", 3, L), ("dense2_b", 4, L)]),
    ("Weights.EncoderLayer", [("mha", 1, "msg:Weights.MHA"), ("ln1_gammas", 2, L),
                              ("ln1_betas", 3, L), ("ffn", 4, "msg:Weights.FFN"),
                              ("ln2_gammas", 5, L), ("ln2_betas", 6, L)]),
    ("Weights.PolicyHead", [("ip_pol_w", 1, L), ("ip_pol_b", 2, L), ("ip2_pol_w", 3, L),
                            ("ip2_pol_b", 4, L), ("ip3_pol_w", 5, L), ("ip3_pol_b", 6, L),
                            ("ip4_pol_w", 7, L), ("pol_encoder", 8, ENC, "rep"),
                            ("pol_headcount", 9, "u32"), ("policy1", 10, CB), ("policy", 11, CB)]),
    ("Weights.ValueHead", [("ip_val_w", 1, L), ("ip_val_b", 2, L), ("ip1_val_w", 3, L),
                           ("ip1_val_b", 4, L), ("ip2_val_w", 5, L), ("ip2_val_b", 6, L),
                           ("ip_val_err_w", 7, L), ("ip_val_err_b", 8, L),
                           ("ip_val_cat_w", 9, L), ("ip_val_cat_b", 10, L), ("value", 11, CB)]),
    ("Weights.PolicyHeadMap", [("key", 1, "str"), ("value", 2, "msg:Weights.PolicyHead")]),
    ("Weights.PolicyHeads", [("ip_pol_w", 1, L), ("ip_pol_b", 2, L),
                             ("vanilla", 3, "msg:Weights.PolicyHead"),
                             ("optimistic_st", 4, "msg:Weights.PolicyHead"),
                             ("soft", 5, "msg:Weights.PolicyHead"),
                             ("opponent", 6, "msg:Weights.PolicyHead"),
                             ("policy_head_map", 7, "msg:Weights.PolicyHeadMap", "rep")]),
    ("Weights.ValueHeadMap", [("key", 1, "str"), ("value", 2, "msg:Weights.ValueHead")]),
    ("Weights.ValueHeads", [("winner", 1, "msg:Weights.ValueHead"), ("q", 2, "msg:Weights.ValueHead"),
                            ("st", 3, "msg:Weights.ValueHead"),
                            ("value_head_map", 4, "msg:Weights.ValueHeadMap", "rep")]),
    ("Weights", [("input", 1, CB), ("residual", 2, "msg:Weights.Residual", "rep"),
                 ("ip_emb_preproc_w", 37, L), ("ip_emb_preproc_b", 38, L),
                 ("ip_emb_w", 25, L), ("ip_emb_b", 26, L), ("ip_emb_ln_gammas", 39, L),
                 ("ip_emb_ln_betas", 40, L), ("ip_mult_gate", 33, L), ("ip_add_gate", 34, L),
                 ("ip_emb_ffn", 41, "msg:Weights.FFN"), ("ip_emb_ffn_ln_gammas", 42, L),
                 ("ip_emb_ffn_ln_betas", 43, L), ("encoder", 27, ENC, "rep"),
                 ("headcount", 28, "u32"), ("pol_encoder", 21, ENC, "rep"),
                 ("pol_headcount", 24, "u32"), ("policy1", 11, CB), ("policy", 3, CB),
                 ("ip_pol_w", 4, L), ("ip_pol_b", 5, L), ("ip2_pol_w", 17, L), ("ip2_pol_b", 18, L),
                 ("ip3_pol_w", 19, L), ("ip3_pol_b", 20, L), ("ip4_pol_w", 22, L),
                 ("value", 6, CB), ("ip_val_w", 29, L), ("ip_val_b", 30, L), ("ip1_val_w", 7, L),
                 ("ip1_val_b", 8, L), ("ip2_val_w", 9, L), ("ip2_val_b", 10, L),
                 ("value_heads", 44, "msg:Weights.ValueHeads"),
                 ("policy_heads", 45, "msg:Weights.PolicyHeads"),
                 ("moves_left", 12, CB), ("ip_mov_w", 31, L), ("ip_mov_b", 32, L),
                 ("ip1_mov_w", 13, L), ("ip1_mov_b", 14, L), ("ip2_mov_w", 15, L),
                 ("ip2_mov_b", 16, L), ("smolgen_w", 35, L), ("smolgen_b", 36, L)]),
    ("TrainingParams", [("training_steps", 1, "u32"), ("learning_rate", 2, "f32"),
                        ("mse_loss", 3, "f32"), ("policy_loss", 4, "f32"), ("accuracy", 5, "f32"),
                        ("network_params", 6, "str")]),
    ("NetworkFormat", [("input", 1, "enum:NetworkFormat.InputFormat"),
                       ("output", 2, "enum:NetworkFormat.OutputFormat"),
                       ("network", 3, "enum:NetworkFormat.NetworkStructure"),
                       ("policy", 4, "enum:NetworkFormat.PolicyFormat"),
                       ("value", 5, "enum:NetworkFormat.ValueFormat"),
                       ("moves_left", 6, "enum:NetworkFormat.MovesLeftFormat"),
                       ("default_activation", 7, "enum:NetworkFormat.DefaultActivation"),
                       ("smolgen_activation", 8, "enum:NetworkFormat.ActivationFunction"),
                       ("ffn_activation", 9, "enum:NetworkFormat.ActivationFunction"),
                       ("input_embedding", 10, "enum:NetworkFormat.InputEmbeddingFormat")]),
    ("Format", [("weights_encoding", 1, "enum:Format.Encoding"),
                ("network_format", 2, "msg:NetworkFormat")]),
    ("OnnxModel", [("model", 1, "bytes"), ("data_type", 2, "enum:OnnxModel.DataType"),
                   ("input_planes", 3, "str"), ("output_value", 4, "str"), ("output_wdl", 5, "str"),
                   ("output_policy", 6, "str"), ("output_mlh", 7, "str")]),
    ("Net", [("magic", 1, "fx32"), ("license", 2, "str"), ("min_version", 3, "msg:EngineVersion"),
             ("format", 4, "msg:Format"), ("training_params", 5, "msg:TrainingParams"),
             ("weights", 10, "msg:Weights"), ("onnx_model", 11, "msg:OnnxModel")]),
]


def cname(dotted):
    return dotted.replace(".", "_")


def enum_owner(dotted):
    return dotted.rsplit(".", 1)[0]


def emit():
    out = []
    w = out.append
    w("// Generated by oracle/shim/gen_net_pb.py -- test infrastructure only.")
    w("// Header-only stand-in for the protobuf classes of the MetalFish weight schema.")
    w("#pragma once")
    w("#include <cstdint>\n#include <cstring>\n#include <deque>\n#include <memory>")
    w("#include <string>\n#include <vector>")
    w('#include "google/protobuf/io/coded_stream.h"')
    w("namespace MetalFishNN {")
    w("namespace wire {")
    w("""inline bool ReadVarint(const std::uint8_t *&p, const std::uint8_t *e, std::uint64_t &v) {
  v = 0; int s = 0;
  while (p < e && s < 64) { std::uint8_t b = *p++; v |= std::uint64_t(b & 0x7f) << s;
    if (!(b & 0x80)) return true; s += 7; }
  return false;
}
inline bool Skip(const std::uint8_t *&p, const std::uint8_t *e, int wt) {
  std::uint64_t v;
  switch (wt) {
  case 0: return ReadVarint(p, e, v);
  case 1: if (e - p < 8) return false; p += 8; return true;
  case 2: if (!ReadVarint(p, e, v) || std::uint64_t(e - p) < v) return false; p += v; return true;
  case 5: if (e - p < 4) return false; p += 4; return true;
  default: return false;
  }
}
inline void PutVarint(std::string &o, std::uint64_t v) {
  while (v >= 0x80) { o.push_back(char((v & 0x7f) | 0x80)); v >>= 7; } o.push_back(char(v));
}
inline void PutTag(std::string &o, int f, int wt) { PutVarint(o, (std::uint64_t(f) << 3) | wt); }
inline void PutFixed32(std::string &o, std::uint32_t v) { char b[4]; std::memcpy(b, &v, 4); o.append(b, 4); }
template <class T> struct Field {
  std::unique_ptr<T> p;
  Field() = default;
  Field(const Field &o) : p(o.p ? std::make_unique<T>(*o.p) : nullptr) {}
  Field &operator=(const Field &o) { p = o.p ? std::make_unique<T>(*o.p) : nullptr; return *this; }
  Field(Field &&) = default;
  Field &operator=(Field &&) = default;
  const T &get() const { static const T empty; return p ? *p : empty; }
  T *mut() { if (!p) p = std::make_unique<T>(); return p.get(); }
};
} // namespace wire""")
    # enums at namespace scope
    for en, vals in ENUMS.items():
        cn = cname(en)
        w(f"enum {cn} : int {{")
        for n, v in vals:
            w(f"  {cn}_{n} = {v},")
        w("};")
    for mname, fields in MESSAGES:
        cn = cname(mname)
        w(f"class {cn} {{\n public:")
        # nested type aliases
        for other, _ in MESSAGES:
            if other.startswith(mname + ".") and other.count(".") == mname.count(".") + 1:
                w(f"  using {other.rsplit('.', 1)[1]} = {cname(other)};")
        for en, vals in ENUMS.items():
            if enum_owner(en) == mname:
                short = en.rsplit(".", 1)[1]
                w(f"  using {short} = {cname(en)};")
                for n, v in vals:
                    w(f"  static constexpr {cname(en)} {n} = {cname(en)}_{n};")
        members = []
        for f in fields:
            name, num, kind = f[0], f[1], f[2]
            rep = len(f) > 3
            if kind.startswith("msg:"):
                t = cname(kind[4:])
                if rep:
                    w(f"  const std::deque<{t}> &{name}() const {{ return {name}_; }}")
                    w(f"  const {t} &{name}(int i) const {{ return {name}_[i]; }}")
                    w(f"  {t} *mutable_{name}(int i) {{ return &{name}_[i]; }}")
                    w(f"  std::deque<{t}> *mutable_{name}() {{ return &{name}_; }}")
                    w(f"  int {name}_size() const {{ return int({name}_.size()); }}")
                    w(f"  {t} *add_{name}() {{ {name}_.emplace_back(); return &{name}_.back(); }}")
                    w(f"  void clear_{name}() {{ {name}_.clear(); }}")
                    members.append(f"  std::deque<{t}> {name}_;")
                else:
                    w(f"  const {t} &{name}() const {{ return {name}_.get(); }}")
                    w(f"  {t} *mutable_{name}() {{ return {name}_.mut(); }}")
                    w(f"  bool has_{name}() const {{ return bool({name}_.p); }}")
                    w(f"  void clear_{name}() {{ {name}_.p.reset(); }}")
                    members.append(f"  wire::Field<{t}> {name}_;")
            elif kind in ("bytes", "str"):
                w(f"  const std::string &{name}() const {{ return {name}_; }}")
                w(f"  void set_{name}(const std::string &v) {{ {name}_ = v; has_{name}_ = true; }}")
                w(f"  void set_{name}(const void *v, std::size_t n) {{ {name}_.assign(static_cast<const char *>(v), n); has_{name}_ = true; }}")
                w(f"  std::string *mutable_{name}() {{ has_{name}_ = true; return &{name}_; }}")
                w(f"  bool has_{name}() const {{ return has_{name}_; }}")
                w(f"  void clear_{name}() {{ {name}_.clear(); has_{name}_ = false; }}")
                members.append(f"  std::string {name}_; bool has_{name}_ = false;")
            else:
                t = {"u32": "std::uint32_t", "f32": "float", "fx32": "std::uint32_t"}.get(kind)
                if kind.startswith("enum:"):
                    t = cname(kind[5:])
                if rep:
                    w(f"  const std::vector<{t}> &{name}() const {{ return {name}_; }}")
                    w(f"  {t} {name}(int i) const {{ return {name}_[i]; }}")
                    w(f"  int {name}_size() const {{ return int({name}_.size()); }}")
                    w(f"  void add_{name}({t} v) {{ {name}_.push_back(v); }}")
                    w(f"  void clear_{name}() {{ {name}_.clear(); }}")
                    members.append(f"  std::vector<{t}> {name}_;")
                else:
                    w(f"  {t} {name}() const {{ return {name}_; }}")
                    w(f"  void set_{name}({t} v) {{ {name}_ = v; has_{name}_ = true; }}")
                    w(f"  bool has_{name}() const {{ return has_{name}_; }}")
                    w(f"  void clear_{name}() {{ {name}_ = {t}(); has_{name}_ = false; }}")
                    members.append(f"  {t} {name}_{{}}; bool has_{name}_ = false;")
        # parser
        w("  bool MergeFromWire(const std::uint8_t *p, const std::uint8_t *e) {")
        w("    while (p < e) {\n      std::uint64_t tag;\n      if (!wire::ReadVarint(p, e, tag)) return false;")
        w("      const int f = int(tag >> 3), wt = int(tag & 7);\n      switch (f) {")
        for f in fields:
            name, num, kind = f[0], f[1], f[2]
            rep = len(f) > 3
            w(f"      case {num}: {{")
            if kind.startswith("msg:") or kind in ("bytes", "str"):
                w("        std::uint64_t n; if (wt != 2 || !wire::ReadVarint(p, e, n) || std::uint64_t(e - p) < n) return false;")
                if kind.startswith("msg:"):
                    if rep:
                        w(f"        if (!add_{name}()->MergeFromWire(p, p + n)) return false;")
                    else:
                        w(f"        if (!mutable_{name}()->MergeFromWire(p, p + n)) return false;")
                else:
                    w(f"        set_{name}(p, std::size_t(n));")
                w("        p += n; break; }")
            elif kind in ("f32", "fx32"):
                t = "float" if kind == "f32" else "std::uint32_t"
                w(f"        if (wt != 5 || e - p < 4) return false; {t} v; std::memcpy(&v, p, 4); p += 4;")
                w(f"        set_{name}(v); break; }}")
            else:
                t = "std::uint32_t" if kind == "u32" else cname(kind[5:])
                if rep:
                    w("        if (wt == 2) { std::uint64_t n; if (!wire::ReadVarint(p, e, n) || std::uint64_t(e - p) < n) return false;")
                    w("          const std::uint8_t *q = p + n; while (p < q) { std::uint64_t v; if (!wire::ReadVarint(p, q, v)) return false;")
                    w(f"            add_{name}({t}(v)); }} break; }}")
                    w(f"        std::uint64_t v; if (wt != 0 || !wire::ReadVarint(p, e, v)) return false; add_{name}({t}(v)); break; }}")
                else:
                    w(f"        std::uint64_t v; if (wt != 0 || !wire::ReadVarint(p, e, v)) return false; set_{name}({t}(v)); break; }}")
        w("      default: if (!wire::Skip(p, e, wt)) return false;\n      }\n    }\n    return true;\n  }")
        # serializer
        w("  void AppendToString(std::string &o) const {")
        for f in sorted(fields, key=lambda x: x[1]):
            name, num, kind = f[0], f[1], f[2]
            rep = len(f) > 3
            if kind.startswith("msg:"):
                if rep:
                    w(f"    for (const auto &m : {name}_) {{ std::string s; m.AppendToString(s); wire::PutTag(o, {num}, 2); wire::PutVarint(o, s.size()); o += s; }}")
                else:
                    w(f"    if ({name}_.p) {{ std::string s; {name}_.p->AppendToString(s); wire::PutTag(o, {num}, 2); wire::PutVarint(o, s.size()); o += s; }}")
            elif kind in ("bytes", "str"):
                w(f"    if (has_{name}_) {{ wire::PutTag(o, {num}, 2); wire::PutVarint(o, {name}_.size()); o += {name}_; }}")
            elif kind == "f32":
                w(f"    if (has_{name}_) {{ wire::PutTag(o, {num}, 5); std::uint32_t b; std::memcpy(&b, &{name}_, 4); wire::PutFixed32(o, b); }}")
            elif kind == "fx32":
                w(f"    if (has_{name}_) {{ wire::PutTag(o, {num}, 5); wire::PutFixed32(o, {name}_); }}")
            else:
                if rep:
                    w(f"    for (auto v : {name}_) {{ wire::PutTag(o, {num}, 0); wire::PutVarint(o, std::uint64_t(v)); }}")
                else:
                    w(f"    if (has_{name}_) {{ wire::PutTag(o, {num}, 0); wire::PutVarint(o, std::uint64_t(std::uint32_t({name}_))); }}")
        w("  }")
        w("  bool SerializeToString(std::string *o) const { o->clear(); AppendToString(*o); return true; }")
        w("  bool ParseFromArray(const void *d, int n) { *this = " + cn + "(); auto *p = static_cast<const std::uint8_t *>(d); return MergeFromWire(p, p + n); }")
        w("  bool ParseFromString(const std::string &s) { return ParseFromArray(s.data(), int(s.size())); }")
        w("  bool ParseFromCodedStream(google::protobuf::io::CodedInputStream *in) {")
        w("    *this = " + cn + "(); auto *p = in->data(); return MergeFromWire(p, p + in->size()); }")
        w(" private:")
        out.extend(members)
        w("};")
    w("} // namespace MetalFishNN")
    return "\n".join(out) + "\n"


CODED = """// Generated by oracle/shim/gen_net_pb.py -- test infrastructure only.
#pragma once
#include <cstddef>
#include <cstdint>
namespace google { namespace protobuf { namespace io {
class ArrayInputStream {
 public:
  ArrayInputStream(const void *data, std::size_t size) : d_(static_cast<const std::uint8_t *>(data)), n_(size) {}
  const std::uint8_t *d_; std::size_t n_;
};
class CodedInputStream {
 public:
  explicit CodedInputStream(ArrayInputStream *s) : s_(s) {}
  void SetTotalBytesLimit(int) {}
  const std::uint8_t *data() const { return s_->d_; }
  std::size_t size() const { return s_->n_; }
 private:
  ArrayInputStream *s_;
};
}}}
"""

ZC = """// Generated by oracle/shim/gen_net_pb.py -- test infrastructure only.
#pragma once
#include "google/protobuf/io/coded_stream.h"
"""

if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__))
    os.makedirs(os.path.join(root, "proto"), exist_ok=True)
    os.makedirs(os.path.join(root, "google/protobuf/io"), exist_ok=True)
    with open(os.path.join(root, "proto/net.pb.h"), "w") as f:
        f.write(emit())
    with open(os.path.join(root, "google/protobuf/io/coded_stream.h"), "w") as f:
        f.write(CODED)
    with open(os.path.join(root, "google/protobuf/io/zero_copy_stream_impl.h"), "w") as f:
        f.write(ZC)
