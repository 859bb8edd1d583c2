//go:build goexperiment.simd && sptcuda

// Package forward, CUDA build of the Q8_0 output head: MulQ80Argmax and
// MulQ80Into call libspt_moe.so (include/spt_moe.h, spt_mul_q80_matrix)
// instead of the Go SIMD kernels.  Build as moe_cuda.go describes and delete
// the two functions' pure-Go definitions from forward/q80.go (20-148); the
// rest of that file (q80Shape, dotQ80, the constants) stays and is used here.
// Signatures, checks and error texts are the reference's; logits are bit for
// bit those of its AVX2 kernels (quantDotQ80Pair / dotQ80), and the argmax
// keeps its rules: largest logit, lowest row on ties, NaN never chosen, row 0
// and -Inf when no logit beats -Inf.
//
// Each tensor is uploaded once into HBM (keyed by the reader and the tensor's
// byte range), repacked there and kept resident, replacing the streamed mmap
// window: options.WindowBytes is checked as before, and neither it nor
// options.Workers (which the reference only clamps) shapes the work.  One
// call is a single device pass of about 0.12 ms for GPT-OSS's head, so ctx is
// checked before and after it.
package forward

/*
#include <stdint.h>
#include <stdlib.h>
#include "spt_moe.h"
*/
import "C"

import (
	"context"
	"fmt"
	"sync"
	"unsafe"

	"Stream-PT/ggufindex"
	ggufmmap "Stream-PT/ggufmap"
)

type q80Key struct {
	reader *ggufmmap.Reader
	rng    ggufindex.Range
}

var (
	sptQ80M sync.Mutex
	sptQ80  = map[q80Key]*C.spt_q80_matrix{}
)

// q80Matrix uploads the tensor once, read through the Reader's own
// WithTensor (ggufmap/mmap_linux.go); the library copies the view while the
// callback runs and keeps nothing of it.
func q80Matrix(ctx *C.spt_context, reader *ggufmmap.Reader, tensor ggufindex.Tensor,
	input, output int) (*C.spt_q80_matrix, error) {
	key := q80Key{reader, tensor.Range}
	sptQ80M.Lock()
	defer sptQ80M.Unlock()
	if m, ok := sptQ80[key]; ok {
		return m, nil
	}
	var m *C.spt_q80_matrix
	err := reader.WithTensor(tensor, func(data []byte) error {
		sptCallM.Lock()
		defer sptCallM.Unlock()
		return sptError(ctx, C.spt_q80_matrix_create(ctx, first(data), C.uint64_t(len(data)),
			C.int64_t(input), C.int64_t(output), &m))
	})
	if err != nil {
		return nil, err
	}
	sptQ80[key] = m
	return m, nil
}

// q80Window is the reference's window check (forward/q80.go:46-52, 122-128).
func q80Window(options Q40Options, rowBytes int) error {
	windowBytes := options.WindowBytes
	if windowBytes == 0 {
		windowBytes = DefaultQ40WindowBytes
	}
	if windowBytes < uint64(rowBytes) {
		return fmt.Errorf("window of %d bytes cannot accommodate a %d-byte row", windowBytes, rowBytes)
	}
	return nil
}

// mulQ80 runs the head on the device: y (nil for the argmax only) and the
// argmax token and logit.
func mulQ80(reader *ggufmmap.Reader, tensor ggufindex.Tensor, input, output int,
	x, y []float32) (int, float32, error) {
	sctx, err := sptContext()
	if err != nil {
		return 0, 0, err
	}
	m, err := q80Matrix(sctx, reader, tensor, input, output)
	if err != nil {
		return 0, 0, err
	}
	var yp *C.float
	if y != nil {
		yp = (*C.float)(unsafe.Pointer(&y[0]))
	}
	var token C.int64_t
	var logit C.float
	sptCallM.Lock()
	st := C.spt_mul_q80_matrix(sctx, m, (*C.float)(unsafe.Pointer(&x[0])), yp, &token, &logit)
	err = sptError(sctx, st)
	sptCallM.Unlock()
	if err != nil {
		return 0, 0, err
	}
	return int(token), float32(logit), nil
}

// MulQ80Argmax: same contract as forward/q80.go:20-105.
func MulQ80Argmax(
	ctx context.Context,
	reader *ggufmmap.Reader,
	tensor ggufindex.Tensor,
	x []float32,
	options Q40Options,
) (bestToken int, bestLogit float32, err error) {
	if ctx == nil {
		return 0, 0, fmt.Errorf("nil context")
	}
	if reader == nil {
		return 0, 0, fmt.Errorf("nil reader")
	}
	if err := ctx.Err(); err != nil {
		return 0, 0, err
	}
	input, output, rowBytes, err := q80Shape(tensor)
	if err != nil {
		return 0, 0, err
	}
	if len(x) != input {
		return 0, 0, fmt.Errorf("%q: expected %d input elements, got %d", tensor.Name, input, len(x))
	}
	if err := q80Window(options, rowBytes); err != nil {
		return 0, 0, err
	}
	bestToken, bestLogit, err = mulQ80(reader, tensor, input, output, x, nil)
	if err != nil {
		return 0, 0, err
	}
	return bestToken, bestLogit, ctx.Err()
}

// MulQ80Into: same contract as forward/q80.go:107-148.
func MulQ80Into(ctx context.Context, reader *ggufmmap.Reader, tensor ggufindex.Tensor, x, y []float32, options Q40Options) error {
	if ctx == nil || reader == nil {
		return fmt.Errorf("nil context or reader")
	}
	if err := ctx.Err(); err != nil {
		return err
	}
	input, output, rowBytes, err := q80Shape(tensor)
	if err != nil {
		return err
	}
	if len(x) != input || len(y) != output {
		return fmt.Errorf("%q: expected input/output lengths %d/%d, got %d/%d", tensor.Name, input, output, len(x), len(y))
	}
	if err := q80Window(options, rowBytes); err != nil {
		return err
	}
	if _, _, err := mulQ80(reader, tensor, input, output, x, y); err != nil {
		return err
	}
	return ctx.Err()
}
