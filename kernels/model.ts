// kernels/model.ts drop-in: embed -> held layers -> output_norm -> tied head
// -> argmax on CUDA through libflock_cuda.so.  One flock_model handle owns
// the uploaded layers (only those below `cut`), the tied table, the KV
// caches and the CUDA graphs; each method is one C-ABI call.  The names,
// argument meaning and thrown errors follow model.ts:65-588 (cut range, hidden
// mismatch, encodePartial's offset check at :438-445).
import { check, flock, FLOCK_DECODE_KERNELS, FLOCK_DECODE_STREAM, handleSlot, pointerArray,
  slotPointer } from "./cuda_ffi.ts";
import { type CudaDevice } from "./lib.ts";
import { configBytes, type LayerConfig, QWEN3_06B, TENSOR_NAMES, uploadF32, uploadQ8 } from "./layer.ts";
import type { RealModel } from "./real_weights.ts";

/** model.ts:65 ModelConfig. */
export interface ModelConfig extends LayerConfig {
  vocab: number;
  nLayers: number;
}

/** How single-token steps run on the device (the kernel graph is the default). */
export type DecodeEngine = "kernels" | "stream";

const ids32 = (ids: number[]) => Int32Array.from(ids);

/** model.ts:70 Model. */
export class Model {
  private freed = false;

  private constructor(
    readonly cfg: ModelConfig,
    readonly handle: Deno.PointerValue,
    private readonly owned: Deno.PointerValue[],
  ) {}

  /**
   * model.ts:109 create(dev, m, base, {cut}): upload layers 0..cut-1 (all by
   * default), the tied token_embd table and output_norm.
   */
  static create(
    dev: CudaDevice,
    m: RealModel,
    base: LayerConfig = QWEN3_06B,
    opts: { cut?: number } = {},
  ): Promise<Model> {
    const cut = opts.cut ?? m.nLayers;
    if (!Number.isInteger(cut) || cut < 0 || cut > m.nLayers) {
      throw new Error(`cut ${cut} is not in 0..${m.nLayers}`);
    }
    const cfg: ModelConfig = { ...base, vocab: m.vocab, nLayers: m.nLayers };
    if (m.hidden !== cfg.hidden) throw new Error(`model hidden ${m.hidden} != config ${cfg.hidden}`);
    if (m.embd.cols !== cfg.hidden) {
      throw new Error(`token_embd cols ${m.embd.cols} != hidden ${cfg.hidden}`);
    }
    const owned: Deno.PointerValue[] = [];
    const layerTensors: Deno.PointerValue[] = [];
    for (let l = 0; l < cut; l++) {
      const w = m.layers[l];
      for (const name of TENSOR_NAMES) {
        let h: Deno.PointerValue;
        if (name in w.f32) h = uploadF32(dev, w.f32[name]);
        else if (name in w.q8) h = uploadQ8(dev, w.q8[name].rows, w.q8[name].cols, w.q8[name].packed);
        else throw new Error(`layer ${l} is missing 1 tensor(s): ${name}`);
        owned.push(h);
        layerTensors.push(h);
      }
    }
    const embd = uploadQ8(dev, m.embd.rows, m.embd.cols, m.embd.packed);
    const onorm = uploadF32(dev, m.outputNorm);
    owned.push(embd, onorm);
    const slot = handleSlot();
    check(flock().flock_model_create(dev.handle, configBytes(cfg), m.vocab, cut,
      pointerArray(layerTensors.length ? layerTensors : [null]), embd, onorm, null, cut, slot));
    return Promise.resolve(new Model(cfg, slotPointer(slot), owned));
  }

  /** model.ts:200 reset: empty every cache, position 0. */
  reset(): void {
    check(flock().flock_model_reset(this.handle));
  }

  /** model.ts:387 step: prefill `ids` (or decode one id), return the next id. */
  step(ids: number[]): Promise<number> {
    const next = new Int32Array(1);
    check(flock().flock_model_step(this.handle, ids32(ids), ids.length, next));
    return Promise.resolve(next[0]);
  }

  /** model.ts:400 logits: the [vocab] logits of the last position. */
  logits(ids: number[]): Promise<Float32Array> {
    const out = new Float32Array(this.cfg.vocab);
    check(flock().flock_model_logits(this.handle, ids32(ids), ids.length, out));
    return Promise.resolve(out);
  }

  /** model.ts:409 hiddenState: the last position's hidden state before output_norm. */
  hiddenState(ids: number[]): Promise<Float32Array> {
    const out = new Float32Array(this.cfg.hidden);
    check(flock().flock_model_hidden_state(this.handle, ids32(ids), ids.length, out));
    return Promise.resolve(out);
  }

  /** model.ts:491 normedState: the same after output_norm. */
  normedState(ids: number[]): Promise<Float32Array> {
    const out = new Float32Array(this.cfg.hidden);
    check(flock().flock_model_normed_state(this.handle, ids32(ids), ids.length, out));
    return Promise.resolve(out);
  }

  /**
   * model.ts:437 encodePartial(ids, offset): [n][hidden] after the held
   * layers; `offset` must equal the caches' position (omitted: unchecked).
   */
  encodePartial(ids: number[], offset?: number): Promise<Float32Array> {
    const out = new Float32Array(ids.length * this.cfg.hidden);
    check(flock().flock_model_encode_partial(this.handle, ids32(ids), ids.length, offset ?? -1, out));
    return Promise.resolve(out);
  }

  /** model.ts:474 projectHidden(flat, seq): output_norm + head on the last row. */
  projectHidden(flat: Float32Array, seq: number): Promise<number> {
    const next = new Int32Array(1);
    check(flock().flock_model_project_hidden(this.handle, flat, seq, next));
    return Promise.resolve(next[0]);
  }

  /** model.ts:546 embed: the dequantised rows of token_embd. */
  embed(ids: number[]): Promise<Float32Array> {
    const out = new Float32Array(ids.length * this.cfg.hidden);
    check(flock().flock_model_embed(this.handle, ids32(ids), ids.length, out));
    return Promise.resolve(out);
  }

  /**
   * model.ts:510 stepsAmortized: K steps behind one readback, for
   * measurement (fixed inputs, so the tokens are not a generation).
   */
  async stepsAmortized(ids: number[]): Promise<number> {
    let tok = 0;
    for (const id of ids) tok = await this.step([id]);
    return tok;
  }

  /**
   * Greedy decode with the chosen id fed back on the device: `n` steps from
   * the token the last step chose, one readback at the end.
   */
  decodeDevice(n: number): Promise<number[]> {
    const out = new Int32Array(Math.max(1, n));
    check(flock().flock_model_decode_device(this.handle, n, out));
    return Promise.resolve(Array.from(out.subarray(0, n)));
  }

  /** model.ts:529 rewind: drop the caches back to nKeys. */
  rewind(nKeys: number): void {
    check(flock().flock_model_rewind(this.handle, nKeys));
  }

  /** model.ts:541 currentToken: the id the device argmax holds. */
  currentToken(): Promise<number> {
    const out = new Int32Array(1);
    check(flock().flock_model_current_token(this.handle, out));
    return Promise.resolve(out[0]);
  }

  /** Keys in the caches (the next position). */
  get pos(): number {
    const n = new Int32Array(1);
    check(flock().flock_model_pos(this.handle, n));
    return n[0];
  }

  /** Layers this model holds (its cut). */
  get held(): number {
    const n = new Int32Array(1);
    check(flock().flock_model_held(this.handle, n));
    return n[0];
  }

  /** Select the single-token engine ("kernels": CUDA graph, the default). */
  set decodeEngine(e: DecodeEngine) {
    check(flock().flock_model_set_decode_mode(this.handle,
      e === "stream" ? FLOCK_DECODE_STREAM : FLOCK_DECODE_KERNELS));
  }

  /**
   * model.ts:572 generate(prompt, maxTokens, {eos, onToken}): greedy, one
   * 4-byte readback per token, stopping before an eos id.  Without onToken
   * the whole loop is one C call.
   */
  async generate(
    prompt: number[],
    maxTokens: number,
    opts: { eos?: number[]; onToken?: (id: number, i: number) => void } = {},
  ): Promise<number[]> {
    const eos = opts.eos ?? [];
    if (!opts.onToken) {
      const out = new Int32Array(Math.max(1, maxTokens));
      const n = new Int32Array(1);
      check(flock().flock_model_generate(this.handle, ids32(prompt), prompt.length, maxTokens,
        ids32(eos.length ? eos : [-1]), eos.length, out, n));
      return Array.from(out.subarray(0, n[0]));
    }
    const stop = new Set(eos);
    const out: number[] = [];
    let next = await this.step(prompt);
    for (let i = 0; i < maxTokens; i++) {
      if (stop.has(next)) break;
      out.push(next);
      opts.onToken(next, i);
      if (out.length >= maxTokens) break;
      next = await this.step([next]);
    }
    return out;
  }

  /** Free the model and everything it uploaded. */
  destroy(): void {
    if (this.freed) return;
    this.freed = true;
    check(flock().flock_model_free(this.handle));
    for (const t of this.owned) check(flock().flock_tensor_free(t));
  }
}
