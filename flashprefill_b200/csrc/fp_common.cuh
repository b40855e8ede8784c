// Problem description shared by the three kernels (pooled keys, block search, sparse
// attention) and the decoding of a "query-block row" work item.
//
// Dense inputs are (B, S, H, D) with arbitrary strides; packed varlen inputs are (T, H, D)
// plus cu_seqlens.  Both are handled as a list of sequences: sequence i starts at token
// `start` (dense: 0, with the batch index as a separate TMA coordinate; varlen:
// cu_seqlens[i]), has `len` tokens and nb = ceil(len / 128) query/key blocks.  Rows of
// the per-head block lists are numbered tile_base + qb, where tile_base is the number of
// blocks of all earlier sequences (the reference's cu_tile_seqlens, varlen:8-18).
#pragma once

#include <stdint.h>

#include "fp_device.cuh"

namespace fpb {

constexpr int kBlock = 128;  // query/key block size (the only one supported)
constexpr int kHeadDim = 128;

struct SeqProblem {
  int varlen;         // 0: dense (B,S,H,D); 1: packed (T,H,D) + cu_seqlens
  int nseq;           // dense: batch size; varlen: number of sequences
  int seqlen;         // dense: S
  int nb_dense;       // dense: ceil(S/128)
  int tiles_ub;       // rows of the per-head list arrays (>= total blocks)
  int cap;            // capacity of one block list (>= nb of every sequence)
  int row_lo, nrows;  // dense: the query blocks [row_lo, row_lo + nrows) of each batch entry are
                      // searched and attended (the others are left alone); varlen: 0, unused
  int q_off;          // dense chunked prefill: key positions before the first query row (the q
                      // and out tensors hold positions [q_off, seqlen)); 0 otherwise
  int hq, hk;
  const int* cu_seqlens;  // varlen: device int32 [nseq+1]
  const int* cu_tile;     // varlen: device int32 [nseq+1], filled by the prep kernel
  uint32_t* err;          // device error word
};

struct SeqInfo {
  int start;      // first token (TMA row coordinate) of the sequence
  int len;        // tokens
  int nb;         // blocks
  int tile_base;  // first list row of the sequence
  int bcoord;     // batch coordinate (dense) or 0
};

// Key block -> (sequence, block), over every block of every sequence (pooled keys).
__device__ __forceinline__ bool decode_block(const SeqProblem& P, int item, SeqInfo& s, int& blk) {
  if (!P.varlen) {
    const int b = item / P.nb_dense;
    if (b >= P.nseq) return false;
    blk = item - b * P.nb_dense;
    s.start = 0;
    s.len = P.seqlen;
    s.nb = P.nb_dense;
    s.tile_base = b * P.nb_dense;
    s.bcoord = b;
    return true;
  }
  const int total = __ldg(P.cu_tile + P.nseq);
  if (item >= total) return false;
  int lo = 0, hi = P.nseq;  // largest lo with cu_tile[lo] <= item (skips empty sequences)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(P.cu_tile + mid) <= item) lo = mid; else hi = mid;
  }
  s.start = __ldg(P.cu_seqlens + lo);
  s.len = __ldg(P.cu_seqlens + lo + 1) - s.start;
  s.tile_base = __ldg(P.cu_tile + lo);
  s.nb = __ldg(P.cu_tile + lo + 1) - s.tile_base;
  s.bcoord = 0;
  blk = item - s.tile_base;
  // a sequence longer than max_seq_len is flagged by the prep kernel and skipped here
  return s.nb <= P.cap;
}

// Work item -> (sequence, query block).  Items are visited latest block first, so the most
// expensive rows (late query blocks see the most key blocks) start first.  Dense problems
// cover the query blocks [row_lo, row_lo + nrows) of every batch entry.
__device__ __forceinline__ bool decode_item(const SeqProblem& P, int item, SeqInfo& s, int& blk) {
  if (!P.varlen) {
    const int b = item / P.nrows;
    if (b >= P.nseq) return false;
    blk = P.row_lo + P.nrows - 1 - (item - b * P.nrows);
    s.start = 0;
    s.len = P.seqlen;
    s.nb = P.nb_dense;
    s.tile_base = b * P.nb_dense;
    s.bcoord = b;
    return true;
  }
  const int total = __ldg(P.cu_tile + P.nseq);
  if (item >= total) return false;
  return decode_block(P, total - 1 - item, s, blk);
}

__device__ __forceinline__ void raise_error(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

}  // namespace fpb
