//go:build goexperiment.simd && sptcuda

// Package forward, CUDA build: forwardMoEBatch calls the sm_100a library
// libspt_moe.so through its C ABI (include/spt_moe.h) instead of the Go SIMD
// kernels.  Build with
//
//	CGO_CFLAGS=-I<repo>/include CGO_LDFLAGS="-L<repo>/stream-pt_b200 -lspt_moe" \
//	GOEXPERIMENT=simd go build -tags sptcuda ./...
//
// and drop this file into forward/ in place of the pure-Go definition of
// forwardMoEBatch (forward/moe_batch.go:78-194); the signature and the error
// behaviour are unchanged, and forwardMoE (forward/moe.go:28-64) reaches it
// as before.
//
// Each layer's MoE tensors are uploaded once into an HBM arena, with both
// the bit-exact CUDA-core layout and the tensor-core layout, read through
// the Reader's own WithTensor (ggufmap/mmap_linux.go:210): the slices are
// handed to the library while their callbacks run, and the library keeps
// nothing of them.  The arena replaces the expert window, hot-expert cache
// and lookahead of WithExpertRanges.  Arenas are keyed by the reader and the
// byte ranges of the layer's tensors, so forwardMoE's per-call LayerWeights
// values reuse the arena of their layer.
package forward

/*
#cgo LDFLAGS: -lspt_moe
#include <stdint.h>
#include <stdlib.h>
#include "spt_moe.h"
*/
import "C"

import (
	"context"
	"errors"
	"fmt"
	"sync"
	"sync/atomic"
	"unsafe"

	"Stream-PT/ggufindex"
	ggufmmap "Stream-PT/ggufmap"
)

// arenaKey identifies a layer's MoE weights: the reader and the byte ranges
// of every tensor the arena holds.
type arenaKey struct {
	reader                                          *ggufmmap.Reader
	router, routerBias, gate, gateBias, up, upBias  ggufindex.Range
	down, downBias, norm                            ggufindex.Range
}

var (
	sptOnce   sync.Once
	sptCtx    *C.spt_context
	sptErr    error
	sptArenaM sync.Mutex
	sptArena  = map[arenaKey]*C.spt_arena{}
	// sptCallM serialises every call into the context (uploads and
	// products): they share its stream, device buffers and error text (the
	// reference gives each caller its own scratch).
	sptCallM sync.Mutex
)

func sptContext() (*C.spt_context, error) {
	sptOnce.Do(func() {
		if st := C.spt_context_create(0, &sptCtx); st != C.SPT_OK {
			sptErr = fmt.Errorf("spt: %s", C.GoString(C.spt_last_error(nil)))
		}
	})
	return sptCtx, sptErr
}

func sptError(ctx *C.spt_context, st C.spt_status) error {
	if st == C.SPT_OK {
		return nil
	}
	if st == C.SPT_ERR_CANCELED {
		return context.Canceled
	}
	return errors.New(C.GoString(C.spt_last_error(ctx)))
}

// sptTensor converts a ggufindex.Tensor; the name is copied into C memory
// that the caller frees.
func sptTensor(t ggufindex.Tensor, names *[]*C.char) C.spt_tensor {
	var c C.spt_tensor
	if t.Name != "" {
		n := C.CString(t.Name)
		*names = append(*names, n)
		c.name = n
	}
	c._type = C.uint32_t(t.Type)
	c.n_dims = C.uint32_t(len(t.Shape))
	for i := 0; i < len(t.Shape) && i < 4; i++ {
		c.shape[i] = C.uint64_t(t.Shape[i])
	}
	c.start, c.end = C.uint64_t(t.Range.Start), C.uint64_t(t.Range.End)
	return c
}

// withTensors opens every named tensor of ts through reader.WithTensor,
// nested, and calls fn with all of their slices (nil for unnamed ones) while
// every mapping is alive.
func withTensors(reader *ggufmmap.Reader, ts []ggufindex.Tensor, views [][]byte, fn func([][]byte) error) error {
	if len(ts) == 0 {
		return fn(views)
	}
	if ts[0].Name == "" {
		return withTensors(reader, ts[1:], append(views, nil), fn)
	}
	return reader.WithTensor(ts[0], func(data []byte) error {
		return withTensors(reader, ts[1:], append(views, data), fn)
	})
}

func first(b []byte) *C.uint8_t {
	if len(b) == 0 {
		return nil
	}
	return (*C.uint8_t)(unsafe.Pointer(&b[0]))
}

// arenaFor uploads the layer once and returns its arena afterwards.
func arenaFor(ctx *C.spt_context, reader *ggufmmap.Reader, cfg *Config, lw *LayerWeights) (*C.spt_arena, error) {
	key := arenaKey{reader, lw.FFNGateInp.Range, lw.FFNGateInpBias.Range, lw.FFNGateExps.Range,
		lw.FFNGateExpsBias.Range, lw.FFNUpExps.Range, lw.FFNUpExpsBias.Range, lw.FFNDownExps.Range,
		lw.FFNDownExpsBias.Range, lw.PostAttnNorm.Range}
	sptArenaM.Lock()
	defer sptArenaM.Unlock()
	if a, ok := sptArena[key]; ok {
		return a, nil
	}
	var names []*C.char
	defer func() {
		for _, n := range names {
			C.free(unsafe.Pointer(n))
		}
	}()
	c := C.spt_moe_config{C.int64_t(cfg.HiddenDim), C.int64_t(cfg.ExpertHiddenDim),
		C.int64_t(cfg.NumExperts), C.int64_t(cfg.NumExpertsUsed)}
	ts := []ggufindex.Tensor{lw.FFNGateInp, lw.FFNGateInpBias, lw.FFNGateExps, lw.FFNGateExpsBias,
		lw.FFNUpExps, lw.FFNUpExpsBias, lw.FFNDownExps, lw.FFNDownExpsBias, lw.PostAttnNorm}
	w := C.spt_layer_weights{
		ffn_gate_inp: sptTensor(ts[0], &names), ffn_gate_inp_bias: sptTensor(ts[1], &names),
		ffn_gate_exps: sptTensor(ts[2], &names), ffn_gate_exps_bias: sptTensor(ts[3], &names),
		ffn_up_exps: sptTensor(ts[4], &names), ffn_up_exps_bias: sptTensor(ts[5], &names),
		ffn_down_exps: sptTensor(ts[6], &names), ffn_down_exps_bias: sptTensor(ts[7], &names),
		post_attention_norm: sptTensor(ts[8], &names),
	}
	var arena *C.spt_arena
	err := withTensors(reader, ts, nil, func(v [][]byte) error {
		// the slices are mmap views, not Go heap memory: C may read them
		// during this call and keeps no reference afterwards
		d := C.spt_layer_data{
			ffn_gate_inp: first(v[0]), ffn_gate_inp_bias: first(v[1]),
			ffn_gate_exps: first(v[2]), ffn_gate_exps_bias: first(v[3]),
			ffn_up_exps: first(v[4]), ffn_up_exps_bias: first(v[5]),
			ffn_down_exps: first(v[6]), ffn_down_exps_bias: first(v[7]),
			post_attention_norm: first(v[8]),
		}
		sptCallM.Lock() // the upload uses the context's stream and error text
		defer sptCallM.Unlock()
		return sptError(ctx, C.spt_arena_create_views(ctx, &c, &w, &d, 1, C.SPT_ARENA_GEMV|C.SPT_ARENA_MMA, 0, 0,
			&arena))
	})
	if err != nil {
		return nil, err
	}
	sptArena[key] = arena
	return arena, nil
}

// forwardMoEBatch: same contract as forward/moe_batch.go:78-194.  x and out
// hold no Go pointers, so passing &x[0] / &out[0] to C is legal; C keeps
// neither after returning (pageable memory is staged through the library's
// pinned buffers).
func forwardMoEBatch(ctx context.Context, reader *ggufmmap.Reader, x []float32, cfg *Config,
	lw *LayerWeights, out []float32, batch int, options Q40Options, scratch *moeBatchScratch,
) error {
	if ctx == nil || reader == nil || cfg == nil || lw == nil {
		return fmt.Errorf("nil MoE context, reader, configuration or weights")
	}
	if err := ctx.Err(); err != nil {
		return err
	}
	if len(x) == 0 || len(out) == 0 {
		return fmt.Errorf("invalid MoE batch dimensions")
	}
	sctx, err := sptContext()
	if err != nil {
		return err
	}
	arena, err := arenaFor(sctx, reader, cfg, lw)
	if err != nil {
		return err
	}
	// The cancel flag lives in C memory: C polls it while a goroutine may set
	// it, so it is written with an atomic store and never through Go memory.
	cancel := (*C.int32_t)(C.calloc(1, C.size_t(unsafe.Sizeof(C.int32_t(0)))))
	stop, exited := make(chan struct{}), make(chan struct{})
	go func() { // context cancellation -> the library's cancel flag
		defer close(exited)
		select {
		case <-ctx.Done():
			atomic.StoreInt32((*int32)(unsafe.Pointer(cancel)), 1)
		case <-stop:
		}
	}()
	sptCallM.Lock()
	st := C.spt_forward_moe_batch(sctx, arena, 0,
		(*C.float)(unsafe.Pointer(&x[0])), C.int64_t(len(x)),
		(*C.float)(unsafe.Pointer(&out[0])), C.int64_t(len(out)),
		C.int64_t(batch), cancel)
	err = sptError(sctx, st) // the context's error text, read before another call replaces it
	sptCallM.Unlock()
	close(stop)
	<-exited // the goroutine no longer touches the flag
	C.free(unsafe.Pointer(cancel))
	return err
}
