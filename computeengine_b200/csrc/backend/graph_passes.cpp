// Conv + BatchNorm (+ Relu / Clip) fusion (see graph_passes.h).
#include "graph_passes.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <memory>
#include <variant>
#include <vector>

#ifdef IE_B200_REFERENCE_HEADERS
#include "core/memory/malloc_allocator.h"
#endif

namespace ie_b200 {
namespace {

ie::Value* value_by_id(ie::Graph& g, ie::ValueId id) {
  for (ie::Value& v : g.values) {
    if (v.id == id) return &v;
  }
  return nullptr;
}

// The constant tensor a value names, or nullptr (graph inputs are not constants).
ie::Tensor* constant_of(ie::Graph& g, ie::ValueId id) {
  const ie::Value* v = value_by_id(g, id);
  if (v == nullptr || v->is_input) return nullptr;
  auto it = g.weights.find(v->name);
  if (it == g.weights.end() || it->second.dtype != ie::DType::F32 || it->second.buffer == nullptr) {
    return nullptr;
  }
  return &it->second;
}

std::vector<size_t> consumers(const ie::Graph& g, ie::ValueId id) {
  std::vector<size_t> out;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    for (ie::ValueId in : g.nodes[i].inputs) {
      if (in == id) {
        out.push_back(i);
        break;
      }
    }
  }
  return out;
}

bool is_graph_output(ie::Graph& g, ie::ValueId id) {
  const ie::Value* v = value_by_id(g, id);
  return v == nullptr || v->is_output;
}

ie::ValueId next_value_id(const ie::Graph& g) {
  ie::ValueId next = 0;
  for (const ie::Value& v : g.values) next = std::max<ie::ValueId>(next, v.id + 1);
  return next;
}

bool name_taken(const ie::Graph& g, const std::string& name) {
  if (g.weights.count(name) != 0) return true;
  for (const ie::Value& v : g.values) {
    if (v.name == name) return true;
  }
  return false;
}

std::string unique_name(const ie::Graph& g, const std::string& base) {
  std::string name = base;
  for (int i = 1; name_taken(g, name); ++i) name = base + "." + std::to_string(i);
  return name;
}

// Adds a constant value + tensor; returns its id.
ie::ValueId add_constant(ie::Graph& g, const std::string& name, ie::Tensor t) {
  ie::Value v;
  v.id = next_value_id(g);
  v.name = name;
  v.shape = t.shape;
  v.dtype = ie::DType::F32;
  g.values.push_back(v);
  g.weights.emplace(name, std::move(t));
  return v.id;
}

// Node `removed` disappears: the value it produced now comes straight from
// node `kept`, the edge carrying kept's output into it goes, and its other
// inputs (an Add's residual) now flow into `kept`.
void splice_out(ie::Graph& g, size_t kept, size_t removed) {
  const ie::NodeId kept_id = g.nodes[kept].id, removed_id = g.nodes[removed].id;
  const ie::ValueId middle = g.nodes[kept].outputs[0];
  g.nodes[kept].outputs = g.nodes[removed].outputs;
  std::vector<ie::Edge> edges;
  for (ie::Edge e : g.edges) {
    if (e.value == middle && e.to.has_value() && *e.to == removed_id) continue;
    if (e.from.has_value() && *e.from == removed_id) e.from = kept_id;
    if (e.to.has_value() && *e.to == removed_id) e.to = kept_id;
    edges.push_back(e);
  }
  g.edges = std::move(edges);
  g.nodes.erase(g.nodes.begin() + static_cast<std::ptrdiff_t>(removed));
}

ie::Result<double> read_number(const ie::Attrs& attrs, const char* key, double dflt) {
  auto it = attrs.find(key);
  if (it == attrs.end()) return dflt;
  if (const auto* d = std::get_if<double>(&it->second)) return *d;
  if (const auto* i = std::get_if<int64_t>(&it->second)) return static_cast<double>(*i);
  return ie::Error::invalid_argument(std::string("attribute '") + key + "' must be numeric");
}

// Folds BatchNorm node `b` into convolution node `c`.  Returns false (no
// change) when the pattern's constants are missing.
ie::Result<bool> fold(ie::Graph& g, size_t c, size_t b) {
  const ie::Node& conv = g.nodes[c];
  const ie::Node& bn = g.nodes[b];
  ie::Tensor* w = constant_of(g, conv.inputs[1]);
  ie::Tensor* bias = conv.inputs.size() >= 3 ? constant_of(g, conv.inputs[2]) : nullptr;
  if (w == nullptr || w->shape.dims.size() != 4 || (conv.inputs.size() >= 3 && bias == nullptr)) {
    return false;
  }
  const int64_t m = w->shape.dims[0];
  if (m <= 0 || (bias != nullptr && bias->numel() != m)) return false;
  const float* p[4];  // scale, bias, mean, var
  for (int i = 0; i < 4; ++i) {
    ie::Tensor* t = constant_of(g, bn.inputs[1 + i]);
    if (t == nullptr) return false;
    if (t->numel() != m) return ie::Error::invalid_argument("BatchNorm parameters must have M values");
    p[i] = t->data<float>();
  }
  auto eps = read_number(bn.attrs, "epsilon", 1e-5);
  if (!eps.has_value()) return eps.error();
  if (*eps < 0.0) return ie::Error::invalid_argument("BatchNorm epsilon must be non-negative");
  auto alloc = std::make_shared<ie::MallocAllocator>();
  auto wf = ie::Tensor::allocate(w->shape, ie::DType::F32, alloc);
  if (!wf.has_value()) return wf.error();
  auto bf = ie::Tensor::allocate(ie::Shape{{m}}, ie::DType::F32, alloc);
  if (!bf.has_value()) return bf.error();
  const int64_t per = w->numel() / m;
  const float* wv = w->data<float>();
  const float* bv = bias != nullptr ? bias->data<float>() : nullptr;
  for (int64_t ch = 0; ch < m; ++ch) {
    const double shifted = static_cast<double>(p[3][ch]) + *eps;
    if (!(shifted > 0.0)) {
      return ie::Error::invalid_argument("BatchNorm variance plus epsilon must be positive");
    }
    const float inv = static_cast<float>(1.0 / std::sqrt(shifted));
    const float gain = p[0][ch] * inv;
    const float mg = p[2][ch] * gain;
    const float shift = p[1][ch] - mg;
    for (int64_t i = 0; i < per; ++i) wf->data<float>()[ch * per + i] = wv[ch * per + i] * gain;
    const float bg = bv != nullptr ? bv[ch] * gain : 0.0f;
    bf->data<float>()[ch] = bg + shift;
  }
  const std::string w_base = value_by_id(g, conv.inputs[1])->name;
  const std::string b_base = bias != nullptr ? value_by_id(g, conv.inputs[2])->name : w_base + ".bias";
  const std::string w_name = unique_name(g, w_base + ".bn_folded");
  const ie::ValueId wid = add_constant(g, w_name, std::move(*wf));
  const std::string b_name = unique_name(g, b_base + ".bn_folded");
  const ie::ValueId bid = add_constant(g, b_name, std::move(*bf));
  ie::Node& conv_node = g.nodes[c];
  conv_node.inputs = {conv_node.inputs[0], wid, bid};
  splice_out(g, c, b);
  return true;
}

// "Relu" for a Relu node, "Relu6" for Clip with attributes min 0 and max 6,
// "Relu" for Clip with min 0 and no max, "" otherwise.
std::string activation_of(const ie::Node& n) {
  if (n.op == ie::OpType::Relu && n.inputs.size() == 1) return "Relu";
  if (n.op == ie::OpType::Clip && n.inputs.size() == 1) {
    auto lo = read_number(n.attrs, "min", -std::numeric_limits<double>::infinity());
    auto hi = read_number(n.attrs, "max", std::numeric_limits<double>::infinity());
    if (lo.has_value() && hi.has_value() && *lo == 0.0) {
      if (*hi == 6.0) return "Relu6";
      if (std::isinf(*hi) && *hi > 0) return "Relu";
    }
  }
  return "";
}

bool is_conv(const ie::Node& n) {
  return n.op == ie::OpType::Conv2D || n.op == ie::OpType::DepthwiseConv2D;
}

// A value the node at `pos` may read: a graph input, a constant, or the
// output of an earlier node.
bool available_at(const ie::Graph& g, ie::ValueId id, size_t pos) {
  for (const ie::Value& v : g.values) {
    if (v.id == id && (v.is_input || g.weights.count(v.name) != 0)) return true;
  }
  for (size_t i = 0; i < pos && i < g.nodes.size(); ++i) {
    for (ie::ValueId o : g.nodes[i].outputs) {
      if (o == id) return true;
    }
  }
  return false;
}

// Conv -> Add(conv, r): r becomes the convolution's fourth input, added in
// its epilogue ("fused_add"); a convolution without a bias gets a zero one.
ie::Result<bool> fuse_add(ie::Graph& g, size_t c, size_t a) {
  const ie::Node& add = g.nodes[a];
  const ie::ValueId out = g.nodes[c].outputs[0];
  if (add.inputs.size() != 2 || add.outputs.size() != 1) return false;
  if (add.inputs[0] == out && add.inputs[1] == out) return false;
  const ie::ValueId r = add.inputs[0] == out ? add.inputs[1] : add.inputs[0];
  if (!available_at(g, r, c)) return false;
  ie::Tensor* w = constant_of(g, g.nodes[c].inputs[1]);
  if (w == nullptr || w->shape.dims.size() != 4) return false;
  if (g.nodes[c].inputs.size() < 3) {
    auto alloc = std::make_shared<ie::MallocAllocator>();
    auto zero = ie::Tensor::allocate(ie::Shape{{w->shape.dims[0]}}, ie::DType::F32, alloc);
    if (!zero.has_value()) return zero.error();
    std::fill(zero->data<float>(), zero->data<float>() + zero->numel(), 0.0f);
    const std::string name = unique_name(g, value_by_id(g, g.nodes[c].inputs[1])->name + ".bias");
    const ie::ValueId bid = add_constant(g, name, std::move(*zero));
    g.nodes[c].inputs.push_back(bid);
  }
  g.nodes[c].inputs.push_back(r);
  g.nodes[c].attrs["fused_add"] = int64_t{1};
  splice_out(g, c, a);
  return true;
}

}  // namespace

ie::Status ConvBnReluFusionPass::run(ie::Graph& graph, ie::PassContext& /*context*/) {
  folded_ = fused_ = fused_adds_ = 0;
  for (size_t i = 0; i < graph.nodes.size(); ++i) {
    if (!is_conv(graph.nodes[i]) || graph.nodes[i].outputs.size() != 1 ||
        graph.nodes[i].inputs.size() < 2) {
      continue;
    }
    // conv -> BatchNorm
    ie::ValueId out = graph.nodes[i].outputs[0];
    auto cons = consumers(graph, out);
    if (cons.size() == 1 && cons[0] > i && !is_graph_output(graph, out)) {
      const ie::Node& n = graph.nodes[cons[0]];
      if (n.op == ie::OpType::BatchNorm && n.inputs.size() == 5 && n.inputs[0] == out &&
          n.outputs.size() == 1) {
        auto r = fold(graph, i, cons[0]);
        if (!r.has_value()) return r.error();
        if (*r) ++folded_;
      }
    }
    // conv -> Add(conv, residual): a dense convolution run by this backend
    if (fuse_activation_ && graph.nodes[i].op == ie::OpType::Conv2D &&
        graph.nodes[i].attrs.count("fused_add") == 0 &&
        graph.nodes[i].attrs.count("activation") == 0) {
      out = graph.nodes[i].outputs[0];
      cons = consumers(graph, out);
      if (cons.size() == 1 && cons[0] > i && !is_graph_output(graph, out) &&
          graph.nodes[cons[0]].op == ie::OpType::Add) {
        auto r = fuse_add(graph, i, cons[0]);
        if (!r.has_value()) return r.error();
        if (*r) ++fused_adds_;
      }
    }
    // conv -> Relu / Clip(0, 6), into a convolution without an activation yet
    if (!fuse_activation_ || graph.nodes[i].attrs.count("activation") != 0) continue;
    out = graph.nodes[i].outputs[0];
    cons = consumers(graph, out);
    if (cons.size() == 1 && cons[0] > i && !is_graph_output(graph, out)) {
      const std::string act = activation_of(graph.nodes[cons[0]]);
      if (!act.empty()) {
        graph.nodes[i].attrs["activation"] = act;
        splice_out(graph, i, cons[0]);
        ++fused_;
      }
    }
  }
  return {};
}

}  // namespace ie_b200
