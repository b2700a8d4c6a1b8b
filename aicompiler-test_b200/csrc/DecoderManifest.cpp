// Decoder manifest import (see DecoderManifest.hpp).
#include "DecoderManifest.hpp"

#include <filesystem>
#include <fstream>
#include <iomanip>
#include <stdexcept>

namespace tensor::importer {
namespace {

void expect(std::istream &in, const char *word) {
  std::string token;
  if (!(in >> token) || token != word)
    throw std::runtime_error(std::string("Expected '") + word + "' in decoder-only manifest.");
}

std::size_t readCount(std::istream &in, const char *what) {
  long long v = -1;
  if (!(in >> v) || v < 0) throw std::runtime_error(std::string("Invalid ") + what + " in decoder-only manifest.");
  return static_cast<std::size_t>(v);
}

std::string readName(std::istream &in, const char *what) {
  std::string v;
  if (!(in >> std::quoted(v))) throw std::runtime_error(std::string("Invalid ") + what + " in decoder-only manifest.");
  return v;
}

bool knownDtype(const std::string &t) { return t == "F32" || t == "F16" || t == "BF16"; }

}  // namespace

const float *DecoderManifest::tensor(const std::string &name, std::size_t *count) const {
  const auto it = ranges.find(name);
  if (it == ranges.end()) {
    if (count) *count = 0;
    return nullptr;
  }
  if (count) *count = it->second.second;
  return payload.data() + it->second.first;
}

std::vector<std::string> decoderWeightNames(std::size_t layers) {
  std::vector<std::string> names = {"embedding.weight", "final_norm.weight", "lm_head.weight", "rope.cosine",
                                    "rope.sine"};
  static const char *kinds[] = {"input_norm", "q", "k", "v", "o", "post_norm", "gate", "up", "down"};
  for (std::size_t l = 0; l < layers; ++l)
    for (const char *k : kinds) names.push_back("layer" + std::to_string(l) + "." + k + ".weight");
  return names;
}

std::string importDecoderManifest(const std::string &path, DecoderManifest *out) {
  try {
    std::ifstream in(path);
    if (!in) throw std::runtime_error("Unable to open decoder-only manifest: " + path);
    DecoderManifest m;
    std::string magic;
    if (!(in >> magic >> m.version) || magic != "TMC_DECODER_LLM" || (m.version != 1 && m.version != 2))
      throw std::runtime_error("Invalid or unsupported decoder-only manifest header.");
    expect(in, "MODEL");
    m.modelName = readName(in, "model name");
    expect(in, "PAYLOAD");
    m.payloadName = readName(in, "payload path");
    expect(in, "CONFIG");
    m.batch = readCount(in, "batch size");
    m.hidden = readCount(in, "hidden size");
    m.heads = readCount(in, "head count");
    if (m.heads == 0 || m.hidden % m.heads != 0)
      throw std::runtime_error("Decoder hidden size must be divisible by head count.");
    m.intermediate = readCount(in, "intermediate size");
    m.vocab = readCount(in, "vocabulary size");
    m.layers = readCount(in, "layer count");
    m.capacity = readCount(in, "cache capacity");
    m.prefillLength = readCount(in, "prefill length");
    m.decodeCount = readCount(in, "decode step count");
    if (!(in >> m.epsilon) || !(m.epsilon > 0.0f)) throw std::runtime_error("Invalid RMSNorm epsilon in decoder-only manifest.");
    if (m.batch == 0 || m.intermediate == 0 || m.vocab == 0 || m.layers == 0 || m.capacity == 0)
      throw std::runtime_error("Decoder-only manifest dimensions must be positive.");
    if (m.prefillLength > m.capacity || m.decodeCount > m.capacity - m.prefillLength)
      throw std::runtime_error("Decoder decode steps exceed cache capacity.");
    m.kvHeads = m.heads;
    std::string marker;
    if (!(in >> marker)) throw std::runtime_error("Missing decoder-only tensor section.");
    if (marker == "ATTENTION") {
      m.kvHeads = readCount(in, "KV head count");
      if (m.kvHeads == 0 || m.heads % m.kvHeads != 0)
        throw std::runtime_error("Decoder KV head count must divide the head count.");
      if (!(in >> m.ropeTheta) || !(m.ropeTheta > 0.0))
        throw std::runtime_error("Invalid RoPE theta in decoder-only manifest.");
      m.attentionLine = true;
      if (!(in >> marker)) throw std::runtime_error("Missing decoder-only tensor section.");
    }
    if (marker == "DTYPE") {
      if (!(in >> m.requestedDtype) || !knownDtype(m.requestedDtype))
        throw std::runtime_error("Unsupported decoder-only dtype.");
      m.effectiveDtype = m.requestedDtype;
      m.dtypeLine = true;
      if (m.version == 2 && (!(in >> m.effectiveDtype) || !knownDtype(m.effectiveDtype)))
        throw std::runtime_error("Unsupported effective decoder-only dtype.");
      if (!(in >> marker)) throw std::runtime_error("Missing decoder-only tensor section.");
    }
    if (marker != "TENSORS") throw std::runtime_error("Expected 'TENSORS' in decoder-only manifest.");
    const std::size_t n = readCount(in, "named tensor count");
    for (std::size_t i = 0; i < n; ++i) {
      expect(in, "TENSOR");
      const std::string name = readName(in, "tensor name");
      const std::size_t offset = readCount(in, "tensor offset"), count = readCount(in, "tensor length");
      if (!m.ranges.emplace(name, std::make_pair(offset, count)).second)
        throw std::runtime_error("Duplicate decoder-only tensor '" + name + "'.");
    }
    expect(in, "END");
    std::string trailing;
    if (in >> trailing) throw std::runtime_error("Unexpected data after decoder-only END marker.");

    const auto payloadPath = std::filesystem::absolute(std::filesystem::path(path)).parent_path() / m.payloadName;
    std::ifstream pin(payloadPath, std::ios::binary | std::ios::ate);
    if (!pin) throw std::runtime_error("Unable to open decoder-only payload: " + payloadPath.string());
    const auto bytes = static_cast<long long>(pin.tellg());
    if (bytes < 0 || bytes % (long long)sizeof(float) != 0)
      throw std::runtime_error("Decoder-only payload is not float32-aligned.");
    m.payload.resize(static_cast<std::size_t>(bytes) / sizeof(float));
    pin.seekg(0);
    if (bytes > 0 && !pin.read(reinterpret_cast<char *>(m.payload.data()), bytes))
      throw std::runtime_error("Unable to read decoder-only payload.");
    for (const auto &r : m.ranges)
      if (r.second.first > m.payload.size() || r.second.second > m.payload.size() - r.second.first)
        throw std::runtime_error("Decoder-only tensor '" + r.first + "' lies outside the payload.");
    *out = std::move(m);
    return {};
  } catch (const std::exception &e) {
    return e.what();
  }
}

}  // namespace tensor::importer
