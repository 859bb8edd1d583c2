//go:build goexperiment.simd && sptcuda

// Package forward, CUDA build: forwardMoEBatch and its stages call the
// sm_100a library libspt_moe.so through its C ABI (include/spt_moe.h)
// instead of the Go SIMD kernels.  Build with
//
//	CGO_CFLAGS=-I<repo>/include CGO_LDFLAGS="-L<repo>/stream-pt_b200 -lspt_moe" \
//	GOEXPERIMENT=simd go build -tags sptcuda ./...
//
// and drop this file into forward/ in place of the pure-Go definitions of
// forwardMoEBatch (forward/moe_batch.go:78-194); the function signature and
// error behaviour are unchanged.  Experts are uploaded once per
// (reader, LayerWeights) into an HBM arena (replacing ggufmap's expert
// window, cache and lookahead) and reused by every later call.
package forward

/*
#cgo LDFLAGS: -lspt_moe
#include <stdlib.h>
#include "spt_moe.h"
*/
import "C"

import (
	"context"
	"errors"
	"fmt"
	"sync"
	"unsafe"

	"Stream-PT/ggufindex"
	ggufmmap "Stream-PT/ggufmap"
)

var (
	sptOnce  sync.Once
	sptCtx   *C.spt_context
	sptErr   error
	sptMu    sync.Mutex
	sptArena = map[*LayerWeights]*C.spt_arena{}
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

// arenaFor uploads the layer once.  The reader's mapped file view is passed
// as the spt_reader (ggufmap exposes it through WithTensor for the whole
// file range).
func arenaFor(ctx *C.spt_context, reader *ggufmmap.Reader, cfg *Config, lw *LayerWeights) (*C.spt_arena, error) {
	sptMu.Lock()
	defer sptMu.Unlock()
	if a, ok := sptArena[lw]; ok {
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
	w := C.spt_layer_weights{
		ffn_gate_inp: sptTensor(lw.FFNGateInp, &names), ffn_gate_inp_bias: sptTensor(lw.FFNGateInpBias, &names),
		ffn_gate_exps: sptTensor(lw.FFNGateExps, &names), ffn_gate_exps_bias: sptTensor(lw.FFNGateExpsBias, &names),
		ffn_up_exps: sptTensor(lw.FFNUpExps, &names), ffn_up_exps_bias: sptTensor(lw.FFNUpExpsBias, &names),
		ffn_down_exps: sptTensor(lw.FFNDownExps, &names), ffn_down_exps_bias: sptTensor(lw.FFNDownExpsBias, &names),
		post_attention_norm: sptTensor(lw.PostAttnNorm, &names),
	}
	var arena *C.spt_arena
	err := reader.WithFile(lw.FFNGateInp.Range.File, func(file []byte) error {
		r := C.spt_reader{base: (*C.uint8_t)(unsafe.Pointer(&file[0])), size: C.uint64_t(len(file))}
		return sptError(ctx, C.spt_arena_create(ctx, &r, &c, &w, 1, C.SPT_ARENA_GEMV, &arena))
	})
	if err != nil {
		return nil, err
	}
	sptArena[lw] = arena
	return arena, nil
}

// forwardMoEBatch: same contract as forward/moe_batch.go:78-194.  x and out
// hold no Go pointers, so passing &x[0] / &out[0] to C is legal; C keeps
// neither after returning.
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
	var cancel C.int32_t
	done := make(chan struct{})
	go func() { // context cancellation -> the library's cancel flag
		select {
		case <-ctx.Done():
			cancel = 1
		case <-done:
		}
	}()
	st := C.spt_forward_moe_batch(sctx, arena, 0,
		(*C.float)(unsafe.Pointer(&x[0])), C.int64_t(len(x)),
		(*C.float)(unsafe.Pointer(&out[0])), C.int64_t(len(out)),
		C.int64_t(batch), &cancel)
	close(done)
	return sptError(sctx, st)
}
