/*
 * The poll bridge of the reference's Apple host (apple/cpu_bridge), with the
 * device token loop of libqwen_b200.so behind it: the same `aie_*` names,
 * codes, event layout and command/event protocol as
 * apple/cpu_bridge/include/llm_cpu_bridge.h, so a caller of that header links
 * this library instead.
 *
 * One model worker at a time (a host thread that owns the model, its
 * generation state and the device session).  Every command is answered by
 * exactly one event, which must be polled before the next command is
 * accepted (AIE_BUSY otherwise).  Inputs are copied during the call; no
 * pointer is retained.
 *
 * Sources (aie_open `kind`):
 *   0  the reference's tiny model JSON (Decoder::from_json, src/model.rs:185;
 *      {"config": ModelConfig, "weights": ModelWeights}, unknown fields
 *      rejected), at most 8 MiB, held as FP32 on the device;
 *   1  a Qwen2 directory (UTF-8 path, at most 4096 bytes) holding config.json
 *      and model.safetensors (BF16), loaded as qb_model_load_safetensors does
 *      with a 32-position context, FP32 on the device, and the chat
 *      tokenizer's tokenizer.json, tokenizer_config.json and
 *      generation_config.json (qb_tokenizer_load_chat): text prompts are
 *      encoded on the worker, generation stops at the tokenizer's stop ids,
 *      and token events carry the stream decoder's text.  The reference also
 *      verifies the files against its pinned inventory hashes; here file
 *      integrity is the caller's.  For tiny models aie_begin_text is
 *      answered by an AIE_INVALID_INPUT event, as in the reference.
 * Models with max_tokens above 32 or a vocabulary above 151,936 are refused
 * (AIE_MODEL_FAILED), as the reference's bridge refuses them.
 */
#ifndef QWEN_B200_BRIDGE_H
#define QWEN_B200_BRIDGE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (llm_cpu_bridge.h:14-18). */
enum {
    AIE_OK = 0, AIE_PENDING = 1, AIE_INVALID_INPUT = 2, AIE_INVALID_HANDLE = 3,
    AIE_BUSY = 4, AIE_CANCELLED = 5, AIE_MODEL_FAILED = 6, AIE_EXECUTION_FAILED = 7,
    AIE_PANIC = 8, AIE_CLOSED = 9
};
/* Event kinds (llm_cpu_bridge.h:19-22). */
enum {
    AIE_READY = 1, AIE_STARTED = 2, AIE_TOKEN = 3, AIE_STOPPED = 4,
    AIE_CANCEL_EVENT = 5, AIE_RESET_EVENT = 6, AIE_ERROR = 7
};
/* llm_cpu_bridge.h:23-28: token = UINT32_MAX for events without one;
 * processed / history are the generation state after the command. */
typedef struct {
    uint32_t kind, code, token, processed, history;
} AieEvent;

/* aie_abi_version, llm_cpu_bridge.h:29: 2. */
uint32_t aie_abi_version(void);
/* aie_open, llm_cpu_bridge.h:35 (src/lib.rs:171-205): returns at once; the
 * worker loads on its own thread and answers with AIE_READY or an AIE_ERROR
 * event (AIE_MODEL_FAILED).  AIE_BUSY while another worker is open or still
 * releasing its model.  On an immediate error *out_handle is unchanged. */
uint32_t aie_open(uint32_t kind, const uint8_t *bytes, size_t length, uint64_t *out_handle);
/* aie_begin_ids, llm_cpu_bridge.h:40 (src/lib.rs:206-226): 1..32 ids,
 * 1 <= max_new < 32; the prompt plus max_new must fit the model's context
 * (8 positions for a Qwen directory), checked on the worker. */
uint32_t aie_begin_ids(uint64_t handle, const uint32_t *ids, size_t count, uint32_t max_new);
/* aie_begin_text, llm_cpu_bridge.h:41 (src/lib.rs:227-247): UTF-8, at most
 * 65,536 bytes; encoded by the source's tokenizer on the worker (a tiny
 * model has none: AIE_INVALID_INPUT). */
uint32_t aie_begin_text(uint64_t handle, const uint8_t *bytes, size_t length, uint32_t max_new);
/* aie_next / aie_reset, llm_cpu_bridge.h:42-43: one greedy token (event
 * AIE_TOKEN, then AIE_STOPPED once stopped) / reset of history, cache and
 * cancellation (AIE_RESET_EVENT). */
uint32_t aie_next(uint64_t handle);
uint32_t aie_reset(uint64_t handle);
/* aie_set_cancel, llm_cpu_bridge.h:46: 1 cancels at token boundaries, 0
 * resumes; takes effect immediately, also during a command. */
uint32_t aie_set_cancel(uint64_t handle, uint32_t enabled);
/* aie_poll, llm_cpu_bridge.h:49 (src/lib.rs:265-287): AIE_OK writes one
 * event and opens command admission; AIE_PENDING and errors write nothing. */
uint32_t aie_poll(uint64_t handle, AieEvent *out_event);
/* aie_poll_text, llm_cpu_bridge.h:56-57 (src/lib.rs:288-323): as aie_poll
 * plus the event's text (a token event's newly decoded text, or "<id> "
 * for a tiny model); `capacity` must be exactly 4096. */
uint32_t aie_poll_text(uint64_t handle, AieEvent *out_event, uint8_t *text, size_t capacity,
                       size_t *out_length);
/* aie_close, llm_cpu_bridge.h:60 (src/lib.rs:324-339): invalidates the handle
 * at once and cancels; the worker frees the model after its current step,
 * and aie_open answers AIE_BUSY until it has. */
uint32_t aie_close(uint64_t handle);

#ifdef __cplusplus
}
#endif
#endif
