// kernels/layer.ts drop-in: one transformer layer on CUDA through
// libflock_cuda.so.  The reference's WebGPU pipelines, bind groups and WGSL
// sources are gone; the layer's weights, activations and KV cache live on
// the CUDA device behind a flock_layer handle, and each encode is one
// flock_layer_encode (a CUDA graph of the layer's kernels).  The exported
// names, argument meaning and thrown errors are the reference's
// (layer.ts:59-801):
//   missing tensors -> "layer is missing N tensor(s): ..." (layer.ts:269-287),
//   KV cache full (:575), maxPrefill overflow (:690-698).
import {
  check,
  cstr,
  flock,
  FLOCK_ATTN_EXACT,
  FLOCK_ATTN_FAST,
  FLOCK_E_UNSUPPORTED,
  FLOCK_KV_BF16,
  FLOCK_KV_FP8,
  FLOCK_MATVEC_EXACT,
  FLOCK_MATVEC_FAST,
  FLOCK_KV_F32,
  FLOCK_PREFILL_EXACT,
  FLOCK_PREFILL_TENSOR,
  FLOCK_Q8_0,
  FLOCK_ROPE_NEOX,
  FLOCK_ROPE_NORM,
  FlockError,
  handleSlot,
  packLayerConfig,
  pointerArray,
  slotPointer,
} from "./cuda_ffi.ts";
import {
  type CommandEncoder,
  type CudaDevice,
  DeviceBuffer,
  type EncodableLayer,
  type LayerPort,
  readBack,
} from "./lib.ts";

export type RopePairing = "norm" | "neox";

/** layer.ts:59: Q8_0 packed straight from the GGUF file, and f32 norm gains. */
export interface LayerWeights {
  q8: Record<string, { rows: number; cols: number; packed: Uint8Array }>;
  f32: Record<string, Float32Array>;
}

/**
 * layer.ts:73: one tensor that is already split into the layout the kernels
 * read.  `qs`/`scales` (Q8_0) or `data` (f32) are host bytes or device
 * buffers; `tensor` is a flock_tensor already on the device (what
 * flock_gguf_load_tensor, the streaming loader, produces), adopted as is.
 */
export interface GpuTensor {
  rows: number;
  cols: number;
  qs?: Uint8Array | DeviceBuffer;
  scales?: Uint8Array | DeviceBuffer;
  data?: Float32Array | DeviceBuffer;
  tensor?: Deno.PointerValue;
}

export type LayerBuffers = Record<string, GpuTensor>;

/**
 * layer.ts:87 LayerConfig, plus the CUDA engine's choices (all optional,
 * defaulting to the reference's arithmetic): `attention` "exact" keeps
 * attnRef's order, "fast" is the split-K flash-decode; `prefill` "tensor"
 * runs multi-token steps on the tcgen05 tensor cores; `kvDtype` "bf16"
 * halves the cache, "fp8" (e4m3) quarters it; `matvec` "fast" runs the decode LM head on the int8
 * tensor cores (reassociated, 1e-3 relative).
 */
export interface LayerConfig {
  hidden: number;
  nHeads: number;
  nKvHeads: number;
  headDim: number;
  ffn: number;
  eps: number;
  ropeBase: number;
  maxKeys: number;
  maxPrefill: number;
  ropePairing: RopePairing;
  attention?: "exact" | "fast";
  prefill?: "exact" | "tensor";
  kvDtype?: "f32" | "bf16" | "fp8";
  matvec?: "exact" | "fast";
}

/** layer.ts:119 QWEN3_06B; maxKeys is not capped by workgroup memory here. */
export const QWEN3_06B: LayerConfig = {
  hidden: 1024,
  nHeads: 16,
  nKvHeads: 8,
  headDim: 128,
  ffn: 3072,
  eps: 9.999999974752427e-7,
  ropeBase: 1e6,
  maxKeys: 2048,
  maxPrefill: 512,
  ropePairing: "neox",
};

/** The 11 tensors a layer needs, in the C ABI's order. */
export const TENSOR_NAMES = [
  "attn_q.weight",
  "attn_k.weight",
  "attn_v.weight",
  "attn_output.weight",
  "ffn_gate.weight",
  "ffn_up.weight",
  "ffn_down.weight",
  "attn_norm.weight",
  "attn_q_norm.weight",
  "attn_k_norm.weight",
  "ffn_norm.weight",
] as const;

const NORMS = new Set<string>(TENSOR_NAMES.slice(7));

/** The flock_layer_config bytes for `cfg`. */
export function configBytes(cfg: LayerConfig): Uint8Array {
  return packLayerConfig({
    hidden: cfg.hidden,
    n_heads: cfg.nHeads,
    n_kv_heads: cfg.nKvHeads,
    head_dim: cfg.headDim,
    ffn: cfg.ffn,
    eps: cfg.eps,
    rope_base: cfg.ropeBase,
    max_keys: cfg.maxKeys,
    max_prefill: cfg.maxPrefill,
    rope_pairing: cfg.ropePairing === "norm" ? FLOCK_ROPE_NORM : FLOCK_ROPE_NEOX,
    attention: cfg.attention === "fast" ? FLOCK_ATTN_FAST : FLOCK_ATTN_EXACT,
    prefill: cfg.prefill === "tensor" ? FLOCK_PREFILL_TENSOR : FLOCK_PREFILL_EXACT,
    kv_dtype: cfg.kvDtype === "bf16" ? FLOCK_KV_BF16 : cfg.kvDtype === "fp8" ? FLOCK_KV_FP8 : FLOCK_KV_F32,
    matvec: cfg.matvec === "fast" ? FLOCK_MATVEC_FAST : FLOCK_MATVEC_EXACT,
  });
}

/**
 * layer.ts:170 wgslSource: there is no WGSL behind this module -- the
 * kernels are CUDA inside libflock_cuda.so -- so asking for a shader's
 * source is an error, not an empty string.
 */
export function wgslSource(file: string): Promise<string> {
  return Promise.reject(
    new FlockError(FLOCK_E_UNSUPPORTED, `${file}: the CUDA build has no WGSL sources`),
  );
}

// --------------------------------------------------------------- tensors

/** Upload one packed Q8_0 tensor (split on the host, bit-exact splitQ8). */
export function uploadQ8(dev: CudaDevice, rows: number, cols: number, packed: Uint8Array): Deno.PointerValue {
  const slot = handleSlot();
  check(flock().flock_tensor_from_packed(dev.handle, FLOCK_Q8_0, packed, rows, cols, slot));
  return slotPointer(slot);
}

/** Upload one f32 vector (a norm gain). */
export function uploadF32(dev: CudaDevice, data: Float32Array): Deno.PointerValue {
  const slot = handleSlot();
  check(flock().flock_tensor_from_f32(dev.handle, data, data.length, slot));
  return slotPointer(slot);
}

async function hostBytes(b: Uint8Array | Float32Array | DeviceBuffer): Promise<Uint8Array> {
  if (b instanceof DeviceBuffer) {
    const f = await readBack(b.dev, b, b.size);
    return new Uint8Array(f.buffer);
  }
  return b instanceof Uint8Array ? b : new Uint8Array(b.buffer, b.byteOffset, b.byteLength);
}

/** A GpuTensor as a flock_tensor handle (adopted, or uploaded from its planes). */
export async function adoptTensor(dev: CudaDevice, name: string, t: GpuTensor): Promise<Deno.PointerValue> {
  if (t.tensor) return t.tensor;
  const slot = handleSlot();
  if (t.qs && t.scales) {
    const qs = await hostBytes(t.qs), sc = await hostBytes(t.scales);
    check(flock().flock_tensor_from_split(dev.handle, FLOCK_Q8_0, qs, sc, t.rows, t.cols, slot));
  } else if (t.data) {
    const bytes = await hostBytes(t.data);
    const f = new Float32Array(bytes.buffer, bytes.byteOffset, t.rows * t.cols || bytes.byteLength / 4);
    check(flock().flock_tensor_from_f32(dev.handle, f, f.length, slot));
  } else {
    throw new Error(`tensor ${name} has neither {qs, scales} nor {data}`);
  }
  return slotPointer(slot);
}

/** Throw the reference's missing-tensor error (layer.ts:269-287). */
export function requireTensors(names: Iterable<string>): void {
  const have = new Set(names);
  const missing = TENSOR_NAMES.filter((n) => !have.has(n));
  if (missing.length) {
    throw new Error(`layer is missing ${missing.length} tensor(s): ${missing.join(", ")}`);
  }
}

// ----------------------------------------------------------------- layer

/** layer.ts:188 Layer. */
export class Layer implements EncodableLayer {
  private freed = false;

  private constructor(
    private readonly dev: CudaDevice,
    readonly cfg: LayerConfig,
    readonly handle: Deno.PointerValue,
    private readonly owned: Deno.PointerValue[],
  ) {}

  private static build(
    dev: CudaDevice,
    cfg: LayerConfig,
    tensors: Map<string, Deno.PointerValue>,
    owned: Deno.PointerValue[],
  ): Layer {
    requireTensors(tensors.keys());
    const names = TENSOR_NAMES.map((n) => cstr(n));
    const namePtrs = pointerArray(names.map((b) => Deno.UnsafePointer.of(b)));
    const ts = pointerArray(TENSOR_NAMES.map((n) => tensors.get(n)!));
    const slot = handleSlot();
    check(flock().flock_layer_create(dev.handle, configBytes(cfg), TENSOR_NAMES.length, namePtrs, ts,
      slot));
    return new Layer(dev, cfg, slotPointer(slot), owned);
  }

  /** layer.ts:228 fromBuffers: adopt tensors already split (or resident). */
  static async fromBuffers(dev: CudaDevice, w: LayerBuffers, cfg: LayerConfig = QWEN3_06B): Promise<Layer> {
    requireTensors(Object.keys(w));
    const tensors = new Map<string, Deno.PointerValue>();
    const owned: Deno.PointerValue[] = [];
    for (const name of TENSOR_NAMES) {
      const h = await adoptTensor(dev, name, w[name]);
      tensors.set(name, h);
      if (!w[name].tensor) owned.push(h);
    }
    return Layer.build(dev, cfg, tensors, owned);
  }

  /** layer.ts:289 create: split each Q8_0 tensor once and upload it. */
  static create(dev: CudaDevice, w: LayerWeights, cfg: LayerConfig = QWEN3_06B): Promise<Layer> {
    requireTensors([...Object.keys(w.q8), ...Object.keys(w.f32)]);
    const tensors = new Map<string, Deno.PointerValue>();
    for (const name of TENSOR_NAMES) {
      if (NORMS.has(name)) tensors.set(name, uploadF32(dev, w.f32[name]));
      else {
        const t = w.q8[name];
        tensors.set(name, uploadQ8(dev, t.rows, t.cols, t.packed));
      }
    }
    return Promise.resolve(Layer.build(dev, cfg, tensors, [...tensors.values()]));
  }

  get hidden(): number {
    return this.cfg.hidden;
  }

  /** Keys in the KV cache (settable, as model.ts:529 rewind sets it). */
  get nKeys(): number {
    const n = new Int32Array(1);
    check(flock().flock_layer_n_keys(this.handle, n));
    return n[0];
  }

  set nKeys(n: number) {
    check(flock().flock_layer_rewind(this.handle, n));
  }

  /** layer.ts:451 reset: empty the KV cache. */
  reset(): void {
    check(flock().flock_layer_reset(this.handle));
  }

  runNow(n: number, hidden: Float32Array | null): void {
    check(flock().flock_layer_encode(this.handle, hidden, n));
  }

  readOutputNow(n: number): Float32Array {
    const out = new Float32Array(n * this.cfg.hidden);
    check(flock().flock_layer_read_output(this.handle, n, out));
    return out;
  }

  readCacheNow(): { k: Float32Array; v: Float32Array } {
    const kv = this.nKeys * this.cfg.nKvHeads * this.cfg.headDim;
    const k = new Float32Array(Math.max(1, kv)), v = new Float32Array(Math.max(1, kv));
    check(flock().flock_layer_read_cache(this.handle, k, v));
    return { k: k.subarray(0, kv), v: v.subarray(0, kv) };
  }

  /** layer.ts:554 forward: one decode step, output read back. */
  forward(hidden: Float32Array): Promise<Float32Array> {
    this.runNow(1, hidden);
    return Promise.resolve(this.readOutputNow(1));
  }

  /** layer.ts:571 encode: one decode step (hidden omitted = already on the device). */
  encode(hidden?: Float32Array, encoder?: CommandEncoder): void {
    if (encoder) encoder.pushLayer(this, 1, hidden ?? null);
    else this.runNow(1, hidden ?? null);
  }

  /** layer.ts:685 encodePrefill: nTokens positions at once. */
  encodePrefill(nTokens: number, hidden?: Float32Array, encoder?: CommandEncoder): void {
    if (encoder) encoder.pushLayer(this, nTokens, hidden ?? null);
    else this.runNow(nTokens, hidden ?? null);
  }

  /** layer.ts:770 outputBuffer / :782 inputBuffer: the activation buffer. */
  outputBuffer(): LayerPort {
    return { layer: this, which: "output" };
  }

  inputBuffer(): LayerPort {
    return { layer: this, which: "input" };
  }

  /** layer.ts:792 cacheBuffers: the K and V caches (readable with readBack). */
  cacheBuffers(): { k: LayerPort; v: LayerPort } {
    return { k: { layer: this, which: "k" }, v: { layer: this, which: "v" } };
  }

  /** layer.ts:801 readOutput. */
  readOutput(nTokens = 1): Promise<Float32Array> {
    return Promise.resolve(this.readOutputNow(nTokens));
  }

  /** Free the layer and the tensors it uploaded. */
  destroy(): void {
    if (this.freed) return;
    this.freed = true;
    check(flock().flock_layer_free(this.handle));
    for (const t of this.owned) check(flock().flock_tensor_free(t));
  }
}
