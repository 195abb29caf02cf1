// Drop-in replacement for the exports of src/bench/webgpu-runtime.js, backed by
// libqdecode.so through the Node-API addon (qdecode.node). Same names, arguments,
// result objects and over-length error as the reference (createWebGpuContext
// :43-60, runKernelBenchmarks :62-96, runFullDecoderStackBenchmark :98-163,
// runCustomQwenGreedyPrompt :165-214).
import { createRequire } from "node:module";

const require = createRequire(import.meta.url);
const native = require("./qdecode.node");

// The reference fetches /qwen/runtime; here it is a directory on disk.
const DEFAULT_RUNTIME = process.env.QDECODE_RUNTIME ?? "public/qwen/runtime";
const DEFAULT_MAX_SEQ = 256;

export async function createWebGpuContext({ runtimeDir = DEFAULT_RUNTIME, device = 0 } = {}) {
  return {
    adapter: { info: { vendor: "nvidia", architecture: "sm_100a" } },
    device: { runtimeDir, ordinal: device, engines: new Map() },
  };
}

function engineFor(device, positions) {
  const cap = Math.max(DEFAULT_MAX_SEQ, positions);
  for (const [c, e] of device.engines) if (c >= positions) return e;
  const e = native.engineCreate(device.runtimeDir, { device: device.ordinal, maxSeq: cap });
  device.engines.set(cap, e);
  return e;
}

export async function runCustomQwenGreedyPrompt({
  device,
  profile,
  inputIds,
  maxNewTokens,
  onToken,
  decodeToken,
  onProgress,
  variant = "optimized", // accepted; every variant runs the one B200 path
  maxSeqLen = DEFAULT_MAX_SEQ,
}) {
  if (inputIds.length + maxNewTokens > maxSeqLen) {
    throw new Error(`Custom CUDA path currently supports prompt + generation length up to ${maxSeqLen} tokens.`);
  }
  void profile; void variant;
  const engine = engineFor(device, inputIds.length + maxNewTokens);
  onProgress?.(`Custom prefill ${inputIds.length}/${inputIds.length}`);
  let step = 0;
  const res = native.generateGreedy(engine, inputIds, maxNewTokens, (id) => {
    step += 1;
    onProgress?.(`Custom decode ${step}/${maxNewTokens}`);
    onToken?.(decodeToken ? decodeToken([id]) : String(id));
  });
  return {
    generated: res.generated,
    generatedTokens: res.generated.length,
    generateMs: res.generateMs,
    firstTokenMs: res.generated.length ? res.firstTokenMs : null,
    outputText: decodeToken ? decodeToken(res.generated) : res.generated.join(" "),
  };
}

function checkProfile(engineProfile, profile) {
  for (const [key, ours] of [["hiddenSize", "hidden"], ["intermediateSize", "intermediate"],
                             ["attentionHeads", "heads"], ["kvHeads", "kvHeads"], ["headDim", "headDim"]]) {
    if (profile?.[key] !== undefined && engineProfile?.[ours] !== undefined && profile[key] !== engineProfile[ours]) {
      throw new Error(`profile.${key}=${profile[key]} does not match the runtime (${engineProfile[ours]})`);
    }
  }
}

export async function runKernelBenchmarks(device, profile) {
  const engine = engineFor(device, 1);
  checkProfile(native.engineProfile(engine), profile);
  return native.kernelBenchmarks(engine);
}

export async function runFullDecoderStackBenchmark(device, profile) {
  const engine = engineFor(device, 1);
  checkProfile(native.engineProfile(engine), profile);
  return native.fullDecoderStackBenchmark(engine);
}
