// Decoder-only model manifests in the reference's export format
// ("TMC_DECODER_LLM 1|2", written by export_decoder_llm.py:554-595 and read by
// importDecoderLLMWorkload, DecoderLLMImporter.cpp:154-281): a text header
//   TMC_DECODER_LLM <version>
//   MODEL "<name>"  PAYLOAD "<file>"
//   CONFIG batch hidden heads intermediate vocab layers capacity prefill decodes epsilon
//   [ATTENTION kv_heads rope_theta]
//   [DTYPE <requested> [<effective> (version 2)]]
//   TENSORS <n>  (TENSOR "<name>" <offset> <count>) x n  END
// and a float32 payload file beside it holding every named tensor (weights by
// the decoder's logical names, RoPE tables, and the exporter's reference
// tokens / logits / KV caches). The same checks as the reference importer:
// heads divide hidden, decode steps fit the cache, no duplicate names, nothing
// after END, a float-aligned payload and every range inside it.
//
// The ATTENTION line is this backend's extension for grouped-query models (the
// reference's descriptors have no KV-head count or RoPE base): kv_heads must
// divide heads, rope_theta must be positive. Without it the model is MHA
// (kv_heads = heads) with the reference exporter's base 10000, so manifests the
// reference writes import unchanged.
#pragma once

#include <cstddef>
#include <map>
#include <string>
#include <utility>
#include <vector>

namespace tensor::importer {

struct DecoderManifest {
  int version = 0;
  std::string modelName, payloadName;
  std::size_t batch = 0, hidden = 0, heads = 0, intermediate = 0, vocab = 0, layers = 0, capacity = 0;
  std::size_t prefillLength = 0, decodeCount = 0;
  float epsilon = 0.0f;
  std::size_t kvHeads = 0;     // = heads unless an ATTENTION line names it
  double ropeTheta = 10000.0;  // RoPE base of the rope.cosine / rope.sine tables
  bool attentionLine = false;
  std::string requestedDtype = "F32", effectiveDtype = "F32";  // F32, F16 or BF16
  bool dtypeLine = false;  // the manifest carries a DTYPE marker
  std::map<std::string, std::pair<std::size_t, std::size_t>> ranges;  // name -> (offset, count) in floats
  std::vector<float> payload;

  // The named tensor, or nullptr (count 0) when absent.
  const float *tensor(const std::string &name, std::size_t *count) const;
};

// Parses `path` and its payload; returns "" or the reason it was rejected.
std::string importDecoderManifest(const std::string &path, DecoderManifest *out);

// The weight names a decoder of `layers` layers loads (embedding, final norm,
// LM head, RoPE tables, and per layer input_norm, q, k, v, o, post_norm, gate,
// up, down).
std::vector<std::string> decoderWeightNames(std::size_t layers);

}  // namespace tensor::importer
