// The Needle-3 engine's interface to the batched decode engine (engine.cu):
// an engine created from a loaded .cact model keeps its per-slot state and
// step buffers in an N3State and runs ndl_forward_batch through n3_forward.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/needle_cuda.h"

namespace ndl {

struct N3State;

int n3_create(const ndl_model *m, int slots, int capacity, int max_rows, int max_heads, cudaStream_t stream,
              N3State **out);
void n3_destroy(N3State *s);
// Validates the rows (slot range, token range, consecutive runs, capacity),
// runs the forward and writes the head rows' logits [heads][vocab].
int n3_forward(N3State *s, cudaStream_t stream, const int *tokens, const int *row_slots, int rows,
               const int *head_rows, int heads, float *logits);
int n3_reset_slot(N3State *s, int slot, cudaStream_t stream);
int n3_slot_length(const N3State *s, int slot);
int n3_slot_mark(const N3State *s, int slot);
int n3_capacity(const N3State *s);
// MarkSlot / RewindSlot on the slot's histories, previous tokens and length.
int n3_mark(N3State *s, int slot, cudaStream_t stream);
int n3_rewind(N3State *s, int slot, cudaStream_t stream);
// The primed-prefix blob of a marked length (the reference's layout with its
// state section) and its moves: export reads the slot's mark, import
// replaces the slot's state, cache, length and mark.
size_t n3_prefix_bytes(const N3State *s, int len);
int n3_prefix_move(N3State *s, int slot, bool to_blob, uint8_t *blob, int len, cudaStream_t stream);
int n3_vocab(const N3State *s);

}  // namespace ndl
