//go:build goexperiment.simd && sptcuda

// Package forward, CUDA build of the Q4_0 products: MulQ40Into and
// MulQ40BatchInto call libspt_moe.so (include/spt_moe.h, spt_mul_q40_matrix)
// instead of the Go SIMD kernels.  Build as moe_cuda.go describes and delete
// the two functions' pure-Go definitions from forward/q40.go (35-101); the
// rest of that file (Q40Options, q40Shape, float32Overlap, the constants)
// stays and is used here.  Signatures, checks and error texts are the
// reference's; results are bit for bit those of its AVX2 kernels
// (quantQ40AVX2 for batch 1, quantDotQ40Batch otherwise).
//
// Each tensor is uploaded once into HBM (keyed by the reader and the
// tensor's byte range) and stays resident, replacing the streamed mmap
// window: options.WindowBytes is checked as before, and neither it nor
// options.Workers (which the reference only clamps) shapes the work.
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
	"sync/atomic"
	"unsafe"

	"Stream-PT/ggufindex"
	ggufmmap "Stream-PT/ggufmap"
)

type q40Key struct {
	reader *ggufmmap.Reader
	rng    ggufindex.Range
}

var (
	sptQ40M sync.Mutex
	sptQ40  = map[q40Key]*C.spt_q40_matrix{}
)

// q40Matrix uploads the tensor once, read through the Reader's own
// WithTensor (ggufmap/mmap_linux.go): the view is handed to the library as a
// one-tensor reader while the callback runs, and the library keeps nothing
// of it.
func q40Matrix(ctx *C.spt_context, reader *ggufmmap.Reader, tensor ggufindex.Tensor) (*C.spt_q40_matrix, error) {
	key := q40Key{reader, tensor.Range}
	sptQ40M.Lock()
	defer sptQ40M.Unlock()
	if m, ok := sptQ40[key]; ok {
		return m, nil
	}
	var names []*C.char
	defer func() {
		for _, n := range names {
			C.free(unsafe.Pointer(n))
		}
	}()
	ct := sptTensor(tensor, &names)
	var m *C.spt_q40_matrix
	err := reader.WithTensor(tensor, func(data []byte) error {
		r := C.spt_reader{base: first(data), size: C.uint64_t(len(data))}
		ct.start, ct.end = 0, C.uint64_t(len(data))
		sptCallM.Lock()
		defer sptCallM.Unlock()
		return sptError(ctx, C.spt_q40_matrix_create(ctx, &r, &ct, &m))
	})
	if err != nil {
		return nil, err
	}
	sptQ40[key] = m
	return m, nil
}

// MulQ40Into writes W*x into y (forward/q40.go:35-40).
func MulQ40Into(ctx context.Context, reader *ggufmmap.Reader, tensor ggufindex.Tensor,
	x, y []float32, options Q40Options) error {
	return MulQ40BatchInto(ctx, reader, tensor, x, y, 1, options)
}

// MulQ40BatchInto: same contract as forward/q40.go:46-101.
func MulQ40BatchInto(ctx context.Context, reader *ggufmmap.Reader, tensor ggufindex.Tensor,
	x, y []float32, batch int, options Q40Options) error {
	if ctx == nil {
		return fmt.Errorf("nil context")
	}
	if reader == nil {
		return fmt.Errorf("nil GGUF reader")
	}
	if err := ctx.Err(); err != nil {
		return err
	}
	input, output, rowBytes, err := q40Shape(tensor)
	if err != nil {
		return err
	}
	maxInt := int(^uint(0) >> 1)
	if batch < 1 || batch > maxInt/input || batch > maxInt/output {
		return fmt.Errorf("invalid or oversized batch: %d", batch)
	}
	if len(x) != batch*input || len(y) != batch*output {
		return fmt.Errorf("%q: expected %d input and %d output elements, got %d and %d",
			tensor.Name, batch*input, batch*output, len(x), len(y))
	}
	if float32Overlap(x, y) {
		return fmt.Errorf("input and output must not overlap")
	}
	windowBytes := options.WindowBytes
	if windowBytes == 0 {
		windowBytes = DefaultQ40WindowBytes
	}
	if windowBytes < uint64(rowBytes) {
		return fmt.Errorf("window of %d bytes cannot accommodate a %d-byte row", windowBytes, rowBytes)
	}
	sctx, err := sptContext()
	if err != nil {
		return err
	}
	m, err := q40Matrix(sctx, reader, tensor)
	if err != nil {
		return err
	}
	// context cancellation -> the library's cancel flag (C memory, atomic store)
	cancel := (*C.int32_t)(C.calloc(1, C.size_t(unsafe.Sizeof(C.int32_t(0)))))
	stop, exited := make(chan struct{}), make(chan struct{})
	go func() {
		defer close(exited)
		select {
		case <-ctx.Done():
			atomic.StoreInt32((*int32)(unsafe.Pointer(cancel)), 1)
		case <-stop:
		}
	}()
	sptCallM.Lock()
	st := C.spt_mul_q40_matrix(sctx, m, (*C.float)(unsafe.Pointer(&x[0])), C.int64_t(len(x)),
		(*C.float)(unsafe.Pointer(&y[0])), C.int64_t(len(y)), C.int64_t(batch), cancel)
	err = sptError(sctx, st)
	sptCallM.Unlock()
	close(stop)
	<-exited
	C.free(unsafe.Pointer(cancel))
	if st == C.SPT_ERR_CANCELED {
		return ctx.Err()
	}
	return err
}
