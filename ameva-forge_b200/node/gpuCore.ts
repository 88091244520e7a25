/**
 * forge_b200 host module: the reference's gpuCore op object and Pyodide bridge
 * surface over the Node-API addon (forge_b200_addon.cc -> libforge_b200.so).
 *
 * Drop-in for packages/forge/src/tensor/gpuCore.ts (op object, :1448-1467) and
 * packages/forge/src/bridge/pyodideBridge.ts (globalThis.amevaForge, :31-58,
 * registerPyodideBridge :105-143): same names, argument order, defaults and
 * Promise-returning calls, so forge-py's bridge (forge-py bridge.py) and the
 * reference's TS callers bind unchanged.  Handles are "tensor_<hex>" strings
 * (types.ts:19); errors are JS Errors whose `name` is the reference's error
 * class (errors.ts:12-111).
 *
 * Ops the C ABI does not serve (training: *_backward, adam_step,
 * sgd_momentum_step, sparseCrossEntropy*) throw AMEVAForgeUnsupportedOpError,
 * as the graph front-end does for them.
 */

export type TensorHandle = string;

export interface TensorInfo {
  handle: TensorHandle;
  shape: number[];
  dtype: string;
  byteLength: number;
  disposed: boolean;
}

export interface QuotaSnapshot {
  limitBytes: number;
  activeBytes: number;
  pendingBytes: number;
  peakBytes: number;
  liveTensors: number;
}

export interface InitOptions {
  device?: number;          // CUDA ordinal
  vramLimitBytes?: number;  // gpuCore.init({vramLimitBytes}) (gpuCore.ts:236-307); 0 = 92 % of free memory
  tpRank?: number;          // tensor parallelism: this process's rank
  tpSize?: number;
  ncclId?: Uint8Array;      // 128 bytes from rank 0
}

interface Addon {
  init(o?: InitOptions): Promise<void>;
  read(h: TensorHandle): Promise<Float32Array>;
  dispose(h: TensorHandle): void;
  disposeBatch(hs: TensorHandle[]): void;
  getTensorInfo(h: TensorHandle): TensorInfo;
  mapBufferAsync(h: TensorHandle): Promise<void>;
  readMappedInto(h: TensorHandle, out: ArrayBufferView): void;
  executeGraph(json: string, inputs: Float32Array[]): Promise<Record<string, TensorHandle>>;
  warmupKernels(): Promise<void>;
  getQuotaSnapshot(): QuotaSnapshot;
  snapshotHandles(): TensorHandle[];
  flushGC(options?: { strict?: boolean }): Promise<{ ok: boolean; error?: string }>;
  configureRuntime(o: Record<string, number | boolean>): void;
  uploadFloat32Array(data: Float32Array, shape: number[]): TensorHandle;
  uploadQuant(type: string, blocks: Uint8Array, rows: number, cols: number): TensorHandle;
  matmul(a: TensorHandle, b: TensorHandle): TensorHandle;
  qmatmul(x: TensorHandle, w: TensorHandle): TensorHandle;
  flashAttention(q: TensorHandle, k: TensorHandle, v: TensorHandle, scale?: number, isCausal?: boolean): TensorHandle;
  rmsNorm(x: TensorHandle, gamma?: TensorHandle, eps?: number): TensorHandle;
  rope(x: TensorHandle, base?: number, offset?: number): TensorHandle;
  swiglu(gate: TensorHandle, up: TensorHandle): TensorHandle;
  add(a: TensorHandle, b: TensorHandle): TensorHandle;
  embedding(w: TensorHandle, idx: TensorHandle): TensorHandle;
  unpackQuant(packed: TensorHandle, scales: TensorHandle, zeros: TensorHandle, bits?: number, groupSize?: number,
              numElements?: number): TensorHandle;
  sample(logits: TensorHandle, temperature?: number, topK?: number, topP?: number, seed?: number): TensorHandle;
  shutdown(): void;
}

// The addon is built next to this file (binding.gyp: build/Release/forge_b200.node).
// eslint-disable-next-line @typescript-eslint/no-var-requires
const addon: Addon = require("./build/Release/forge_b200.node");

function unsupported(name: string): never {
  const e = new Error(`${name} is a training op; forge_b200 serves the inference path only`);
  e.name = "AMEVAForgeUnsupportedOpError";
  throw e;
}

// ---- lifecycle and tensors (gpuCore.ts:236-660) ------------------------------
export const init = (options?: InitOptions): Promise<void> => addon.init(options);
export const read = (handle: TensorHandle): Promise<Float32Array> => addon.read(handle);
export const dispose = (handle: TensorHandle): void => addon.dispose(handle);
export const disposeBatch = (handles: TensorHandle[]): void => addon.disposeBatch(handles);
export const getTensorInfo = (handle: TensorHandle): TensorInfo => addon.getTensorInfo(handle);
export const mapBufferAsync = (handle: TensorHandle): Promise<void> => addon.mapBufferAsync(handle);
export const readMappedInto = (handle: TensorHandle, outArray: ArrayBufferView): void =>
  addon.readMappedInto(handle, outArray);
export const warmupKernels = (): Promise<void> => addon.warmupKernels();
export const getQuotaSnapshot = (): QuotaSnapshot => addon.getQuotaSnapshot();
export const uploadFloat32Array = (data: Float32Array, shape: number[]): TensorHandle =>
  addon.uploadFloat32Array(data, shape);
/** GGUF weight upload (Q4_0 / Q8_0 / Q4_K / Q6_K blocks of a row-major [rows, cols] matrix). */
export const uploadQuant = (type: "Q4_0" | "Q8_0" | "Q4_K" | "Q6_K", blocks: Uint8Array, rows: number,
                            cols: number): TensorHandle => addon.uploadQuant(type, blocks, rows, cols);

// ---- graph front-end (graphExecutor.ts:98-127, 489) ---------------------------
// Graphs run one at a time, in call order, as the reference's promise chain
// serialises them (graphExecutor.ts:487-515).
let _graphChain: Promise<unknown> = Promise.resolve();
export function executeGraph(instructionsJson: string, inputs: Float32Array[]): Promise<Record<string, TensorHandle>> {
  const run = _graphChain.then(() => addon.executeGraph(instructionsJson, inputs));
  _graphChain = run.catch(() => undefined);
  return run;
}
export const configureRuntime = (options: {
  allowNonFinite?: boolean; maxInstructions?: number; maxShapeDim?: number; maxElements?: number;
}): void => addon.configureRuntime(options as Record<string, number | boolean>);

// ---- ops (gpuCore.ts:1448-1467) ----------------------------------------------
export const matmul = (a: TensorHandle, b: TensorHandle): TensorHandle => addon.matmul(a, b);
export const matmulTiled = (a: TensorHandle, b: TensorHandle): TensorHandle => addon.matmul(a, b);
/** nn.Linear over a quantized weight (forge-py nn.py:248-259): x [..., K] @ W[N, K]^T, dequant fused. */
export const qmatmul = (x: TensorHandle, w: TensorHandle): TensorHandle => addon.qmatmul(x, w);
export const flashAttention = (q: TensorHandle, k: TensorHandle, v: TensorHandle, scale?: number,
                               isCausal = false): TensorHandle => addon.flashAttention(q, k, v, scale, isCausal);
export const rmsNorm = (x: TensorHandle, gamma?: TensorHandle, eps = 1e-5): TensorHandle =>
  addon.rmsNorm(x, gamma, eps);
export const rope = (x: TensorHandle, base = 1e4, offset = 0): TensorHandle => addon.rope(x, base, offset);
export const swiglu = (gate: TensorHandle, up: TensorHandle): TensorHandle => addon.swiglu(gate, up);
export const add = (a: TensorHandle, b: TensorHandle): TensorHandle => addon.add(a, b);
export const embedding = (w: TensorHandle, idx: TensorHandle): TensorHandle => addon.embedding(w, idx);
export const unpackQuant = (packed: TensorHandle, scales: TensorHandle, zeros: TensorHandle, bits = 4,
                            groupSize = 128, numElements?: number): TensorHandle =>
  addon.unpackQuant(packed, scales, zeros, bits, groupSize, numElements ?? -1);
/** LLMSampler.sample (sampling.ts:35-128) on the device: I32 handle of the chosen id per row. */
export const sample = (logits: TensorHandle, opts: { temperature?: number; topK?: number; topP?: number;
                                                     seed?: number } = {}): TensorHandle =>
  addon.sample(logits, opts.temperature ?? 1.0, opts.topK ?? 0, opts.topP ?? 1.0, opts.seed);

export const gpuCore = {
  add,
  mul: (_a: TensorHandle, _b: TensorHandle): TensorHandle => unsupported("mul (use the graph front-end)"),
  matmul,
  matmulTiled,
  flashAttention,
  rmsNorm,
  rope,
  swiglu,
  unpackQuant,
  embedding,
  embedding_backward: (): never => unsupported("embedding_backward"),
  adam_step: (): never => unsupported("adam_step"),
  sgd_momentum_step: (): never => unsupported("sgd_momentum_step"),
  sparseCrossEntropy: (): never => unsupported("sparseCrossEntropy"),
  sparseCrossEntropyBackward: (): never => unsupported("sparseCrossEntropyBackward"),
  relu: (_x: TensorHandle): TensorHandle => unsupported("relu (use the graph front-end)"),
  relu_backward: (): never => unsupported("relu_backward"),
  transpose: (_x: TensorHandle): TensorHandle => unsupported("transpose (use the graph front-end)"),
  qmatmul,
  sample,
};

// ---- the Pyodide bridge object (pyodideBridge.ts:31-58, 105-143) --------------
export interface AmevaTensorGlobalAPI {
  init: typeof init;
  read: typeof read;
  dispose: typeof dispose;
  getTensorInfo: typeof getTensorInfo;
  mapBufferAsync: typeof mapBufferAsync;
  readMappedInto: typeof readMappedInto;
  executeGraph: typeof executeGraph;
  warmupKernels: typeof warmupKernels;
  disposeBatch: (handles: TensorHandle[]) => void;
  getQuotaSnapshot: typeof getQuotaSnapshot;
  snapshotHandles: () => string[];
  flushGC: (options?: { strict?: boolean }) => Promise<{ ok: boolean; error?: string }>;
}

declare global {
  // eslint-disable-next-line no-var
  var amevaForge: AmevaTensorGlobalAPI | undefined;
}

export function registerPyodideBridge(): AmevaTensorGlobalAPI {
  const api: AmevaTensorGlobalAPI = {
    init,
    read,
    dispose,
    getTensorInfo,
    mapBufferAsync,
    readMappedInto,
    executeGraph,
    warmupKernels,
    disposeBatch,
    getQuotaSnapshot,
    snapshotHandles: () => addon.snapshotHandles(),
    flushGC: async (options?: { strict?: boolean }) => {
      try {
        return await addon.flushGC(options);
      } catch (e) {
        if (options && options.strict) throw e;
        return { ok: false, error: String(e) };
      }
    },
  };
  Object.freeze(api);
  globalThis.amevaForge = api;
  return api;
}
